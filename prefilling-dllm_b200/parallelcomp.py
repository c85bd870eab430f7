"""GPU-native runtime with the public interface of the reference's `FastDLLMParallelComp`.

Reference: prefilling_dllm_eval/fastdllm_parallelcomp.py — config dataclass :43-110, result dataclasses :113-142,
`split_token_chunks` :158-180, class `FastDLLMParallelComp` :368 with `select_chunks` :1857, `build_prefill_cache`
:2201, `generate_from_cache` :2678, `generate_full_prompt_mask` :2776, `generate` :3026, `generate_from_text_parts`
:3093, factory `load_fastdllm_parallelcomp` :3113. Same names, arguments, result fields and exception types; the
algorithm steps (chunk BOS truncation, draft rounds, label set of the self-information score, stable top-K, keep
lists, RoPE position modes, dual-cache block denoising) follow the reference line by line in BEHAVIOUR, but the
machinery is different: KV lives in a paged pool instead of per-call tensor lists, evicted tokens are dropped by the
slot mapping of the page write, every model call is a packed var-len forward over the sm_100a kernels, and the
sampling / scoring tails are single fused kernels (`ops.unmask_step`, `ops.self_information_scores`, ...).

Where the reference hands tensors around (`past_key_values`), this class hands a `PagedCache` handle.
The default flags run on the fused kernels. Flags off the default path — sampling with temperature / top-p / top-k, the
`topk_margin` / `entropy` confidence rules, `alg_temp`, avg-pooling and the other head / layer reductions, the chunk→query score
direction, the `attention` / `next_block_logits` / per-chunk-draft score modes — reuse the same forwards and finish with a few
device-side torch ops on [rows, vocab] or [heads, chunk] tensors instead of a fused tail.
`model_backend="llada"` (un-shifted read-out, leave-one-out chunk scores) is built for the joint-prefill cache modes without token
eviction: the reference's LLaDA model takes no position ids, so a key's position is its index in the concatenated cache, which
equals this runtime's explicit positions only there.
Not built (raise NotImplementedError): the LLaDA backend with chunk-local caches or token eviction.
"""

from __future__ import annotations

import json
import math
import os
import time
from dataclasses import dataclass, field, fields, is_dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import ops
from .model import DreamArch, PagedDreamModel, denoise_blocks, slots_for


@dataclass
class FastDLLMParallelCompConfig:
    """Field-for-field the reference's config (fastdllm_parallelcomp.py:43-110)."""

    fastdllm_dream_dir: str
    pretrained: str
    model_backend: str = "dream"
    fastdllm_llada_dir: Optional[str] = None
    device: str = "cuda"
    dtype: str = "auto"
    trust_remote_code: bool = True
    llada_score_batch_size: int = 8

    max_new_tokens: int = 32
    max_length: int = 4096
    block_length: int = 32
    diffusion_steps: Optional[int] = None
    temperature: float = 0.0
    top_p: Optional[float] = None
    top_k: Optional[int] = None
    alg: str = "confidence_threshold"
    alg_temp: Optional[float] = 0.0
    threshold: float = 0.9
    add_bos_token: bool = True
    rope_scale_factor: float = 1.0
    rope_scaling_type: str = "yarn"

    chunk_size: int = 1024
    topk_chunks: int = 4
    keep_first_chunk: bool = False
    split_from_tail: bool = False
    chunk_bos: bool = True
    force_keep_chunk_bos: bool = True
    cache_build_mode: str = "chunk_query"

    score_mode: str = "draft_self_information"
    score_query_window: int = 0
    score_draft_tokens: int = 16
    score_draft_steps: Optional[int] = None
    score_draft_fixed_steps: bool = False
    score_draft_partial_steps: Optional[int] = None
    score_draft_partial_rounds: Optional[int] = None
    score_draft_score_all_slots: bool = False
    score_llada_shift_logits: bool = False
    score_attention_mask: str = "causal"
    score_context_mode: str = "single_chunk"
    score_batch_size: int = 8
    attention_score_layers: int = 4
    attention_query_window: int = 0

    token_capacity: int = 0
    token_score_query_window: int = 8
    token_score_layers: int = 0
    token_score_layer_mode: str = "all"
    token_score_reduce: str = "sum"
    token_score_pooling: str = "maxpool"
    token_score_pool_kernel: int = 7
    token_score_head_reduce: str = "sum"
    token_score_layer_reduce: str = "mean"
    token_score_direction: str = "query_to_chunk"
    token_score_keep: str = "high"
    token_score_include_prefix: bool = True
    token_attention_mask: str = "causal"
    token_score_use_generated: bool = False
    token_eviction_granularity: str = "global"

    chunk_position_mode: str = "reuse"
    chunk_query_position_mode: str = "after_reused_window"
    query_position_mode: str = "after_reused_window"
    generation_position_mode: str = "after_query"

    # not in the reference: size of the paged KV pool (pages of 256 tokens); 0 = derive from max_length
    num_kv_pages: int = 0
    decode_cuda_graph: bool = True   # replay the denoise step (forward + unmask) of a block as a CUDA graph


@dataclass
class FastDLLMChunkMeta:
    chunk_index: int
    original_tokens: int
    kept_tokens: int
    removed_tokens: int
    cache_start: int
    cache_end: int
    rope_start: int
    rope_end: int
    score: Optional[float] = None
    kept_positions: List[int] = field(default_factory=list)


@dataclass
class FastDLLMParallelCompResult:
    text: str
    sequences: List[int]
    selected_chunk_indices: List[int]
    chunk_scores: Dict[int, float]
    cache_build_mode: str
    prefix_tokens: int
    query_tokens: int
    raw_context_tokens: int
    candidate_chunks: int
    cache_tokens: int
    removed_tokens: int
    chunk_meta: List[FastDLLMChunkMeta]
    generation_blocks: int
    generation_block_length: int


def dataclass_to_jsonable(obj):
    if is_dataclass(obj):
        return {f.name: dataclass_to_jsonable(getattr(obj, f.name)) for f in fields(obj)}
    if isinstance(obj, dict):
        return {k: dataclass_to_jsonable(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return [dataclass_to_jsonable(v) for v in obj]
    return obj


def split_token_chunks(token_ids: Sequence[int], chunk_size: int, split_from_tail: bool = False) -> List[List[int]]:
    """Fixed-size split; with `split_from_tail` a leading remainder chunk (reference :158-180)."""
    ids = list(token_ids)
    if not ids:
        return []
    if chunk_size <= 0 or len(ids) <= chunk_size:
        return [ids]
    out: List[List[int]] = []
    start = len(ids) % chunk_size if split_from_tail else 0
    if start:
        out.append(ids[:start])
    out.extend(ids[i:i + chunk_size] for i in range(start, len(ids), chunk_size))
    return out


def sample_tokens(logits: torch.Tensor, temperature: float = 0.0, top_p: Optional[float] = None, top_k: Optional[int] = None,
                  margin_confidence: bool = False, neg_entropy: bool = False, generator: Optional[torch.Generator] = None):
    """(confidence, token) per row of `logits` [rows, vocab] — the reference's sampler (fastdllm_parallelcomp.py:183-233) on the
    device the logits live on. Order of the filters as there: temperature, nucleus (keep the smallest prefix of the sorted
    distribution whose mass exceeds top_p, the first token always), top-k (drop what is below the k-th largest), softmax in the
    logits' dtype; greedy arg-max at temperature 0, otherwise one categorical draw (from `generator` when given).
    Confidence: the chosen token's probability, or top-1 minus top-2 probability, or the negative entropy sum p*log(p + 1e-10)."""
    if temperature and temperature > 0:
        logits = logits / temperature
    floor = torch.finfo(logits.dtype).min
    if top_p is not None and top_p < 1:
        ordered, order = torch.sort(logits, dim=-1, descending=True)
        mass = torch.cumsum(torch.softmax(ordered, dim=-1), dim=-1)
        drop_sorted = mass > top_p
        drop_sorted = torch.cat([torch.zeros_like(drop_sorted[..., :1]), drop_sorted[..., :-1]], dim=-1)   # shift right: keep the crossing token
        drop = torch.zeros_like(drop_sorted).scatter(-1, order, drop_sorted)
        logits = logits.masked_fill(drop, floor)
    if top_k is not None:
        kth = torch.topk(logits, min(int(top_k), logits.size(-1)), dim=-1).values[..., -1:]
        logits = logits.masked_fill(logits < kth, floor)
    probs = torch.softmax(logits, dim=-1)
    if temperature and temperature > 0:
        flat = probs.reshape(-1, probs.size(-1)).float()
        token = torch.multinomial(flat, 1, generator=generator).reshape(probs.shape[:-1])
        confidence = torch.gather(probs, -1, token.unsqueeze(-1)).squeeze(-1)
    else:
        confidence, token = probs.max(dim=-1)
    if margin_confidence:
        top2 = torch.topk(probs, 2, dim=-1).values
        confidence = top2[..., 0] - top2[..., 1]
    if neg_entropy:
        confidence = torch.sum(probs * torch.log(probs + 1e-10), dim=-1)
    return confidence, token


_NOT_SCORED = object()      # "no precomputed head scores": distinct from None, which means "nothing could be scored"


class PagedCache:
    """Handle to a request's KV in the paged pool: logical token order → pages, plus the RoPE position of each token."""

    def __init__(self, runtime: "FastDLLMParallelComp", capacity_tokens: int):
        self.model = runtime.model
        n_pages = max(1, math.ceil(capacity_tokens / self.model.page_size))
        self.model.allocator.ensure_free(n_pages)
        self.page_ids: List[int] = self.model.allocator.allocate_pages(n_pages)
        self.length = 0                    # tokens currently valid
        self.positions: List[int] = []     # RoPE position of every valid token
        self._table = self.model.i32(self.page_ids).view(1, -1)
        self.released = False

    @property
    def capacity(self) -> int:
        return len(self.page_ids) * self.model.page_size

    def slots(self, start: int, n: int) -> List[int]:
        if start + n > self.capacity:
            raise RuntimeError(f"paged cache overflow: need {start + n} tokens, capacity {self.capacity}")
        return slots_for(self.page_ids, start, n, self.model.page_size)

    def table(self) -> torch.Tensor:
        return self._table

    def release(self) -> None:
        if not self.released:
            self.model.allocator.release_pages(self.page_ids)
            self.released = True


class _SimpleTokenizer:
    """Stand-in when the checkpoint ships no tokenizer files: ids only."""

    def __init__(self, arch: DreamArch):
        self.bos_token_id = arch.bos_token_id
        self.eos_token_id = arch.eos_token_id
        self.mask_token_id = arch.mask_token_id
        self.eos_token = None
        self.bos_token = None

    def encode(self, text, add_special_tokens=False):
        raise NotImplementedError("this checkpoint has no tokenizer; pass token ids")

    def decode(self, ids, skip_special_tokens=False):
        return " ".join(str(int(i)) for i in ids)


class FastDLLMParallelComp:
    def __init__(self, config: FastDLLMParallelCompConfig, model: Optional[PagedDreamModel] = None, tokenizer=None):
        self.config = config
        self.model_backend = (config.model_backend or "dream").lower()
        if self.model_backend not in {"dream", "llada"}:
            raise ValueError(f"Unsupported model_backend: {config.model_backend}")
        if not torch.cuda.is_available():
            raise RuntimeError("FastDLLMParallelComp (B200) needs a CUDA device; there is no CPU path")
        self.device = torch.device(config.device if str(config.device).startswith("cuda") else "cuda")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.max_new_tokens = int(config.max_new_tokens)
        self.block_length = int(config.block_length)
        if self.max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be positive")
        if self.block_length <= 0:
            raise ValueError("block_length must be positive")
        self.diffusion_steps = int(config.diffusion_steps) if config.diffusion_steps is not None else max(
            1, math.ceil(self.max_new_tokens / self.block_length))
        if config.token_score_direction not in {"query_to_chunk", "chunk_to_query", "bidirectional"}:
            raise ValueError(f"Unsupported token_score_direction: {config.token_score_direction}")
        if config.token_score_keep not in {"high", "low"}:
            raise ValueError(f"Unsupported token_score_keep: {config.token_score_keep}")
        if config.token_eviction_granularity not in {"global", "per_head"}:
            raise ValueError(f"Unsupported token_eviction_granularity: {config.token_eviction_granularity}")
        # one generator per runtime for the sampled paths (temperature > 0, alg_temp > 0); seed it with `manual_seed`
        self.sampling_generator: Optional[torch.Generator] = None
        if self.model_backend == "llada" and (int(config.token_capacity or 0) > 0 or config.cache_build_mode not in {"full_prompt_mask", "full_prompt_query"}):
            # the reference's LLaDA model takes no position ids: a key's RoPE position is its index in the concatenated cache,
            # which equals this runtime's positions only for a jointly prefilled, un-evicted prompt
            raise NotImplementedError("model_backend='llada' is built for the joint-prefill cache modes without token eviction")

        if model is None:
            dtype = _resolve_dtype(config.dtype)
            arch = DreamArch.from_pretrained(config.pretrained)
            if self.model_backend == "llada":
                arch.logit_shift = False
            if dtype in (None, "auto"):
                dtype = torch.bfloat16
            pages = int(config.num_kv_pages) or (4 * math.ceil((config.max_length + config.max_new_tokens) / 256) + 8)
            model = PagedDreamModel.from_pretrained(config.pretrained, device=self.device, dtype=dtype, num_pages=pages, arch=arch)
        self.model = model
        self.arch = model.arch
        if float(config.rope_scale_factor or 1.0) > 1.0:
            kind = (config.rope_scaling_type or "yarn").lower()
            if self.model_backend == "llada" and kind not in {"linear", "yarn"}:
                raise ValueError(f"Unsupported LLaDA RoPE scaling type: {config.rope_scaling_type}")     # reference :560-561
            if self.model_backend == "llada" and kind == "linear":
                model.apply_linear_rope_scaling(float(config.rope_scale_factor))                          # reference :555-690
            elif self.model_backend == "llada":
                # the LLaDA rotary module measures the correction range against `max_sequence_length` (4096 when absent), :566, :645
                original = 4096
                try:
                    with open(os.path.join(config.pretrained or "", "config.json")) as handle:
                        original = int(json.load(handle).get("max_sequence_length") or 4096)
                except (OSError, ValueError):
                    pass
                model.apply_yarn_rope_scaling(float(config.rope_scale_factor), original_max_position_embeddings=original)   # reference :583-617
            else:
                model.apply_yarn_rope_scaling(float(config.rope_scale_factor))                            # reference :539-553
        if tokenizer is None:
            tokenizer = _load_tokenizer(config.pretrained, config.trust_remote_code) or _SimpleTokenizer(self.arch)
        self.tokenizer = tokenizer
        self.generated_token_num = 0
        self.total_generation_time = 0.0

    # ------------------------------------------------------------------------------------------------ small helpers
    def _mask_token_id(self) -> int:
        mask = getattr(self.tokenizer, "mask_token_id", None)
        if mask is None:
            mask = self.arch.mask_token_id
        if mask is None:
            raise ValueError(f"Fast-dLLM {self.model_backend} mask_token_id is not available")
        return int(mask)

    def _get_bos_token_ids(self) -> List[int]:
        bos = getattr(self.tokenizer, "bos_token_id", None)
        if bos is not None:
            return [int(bos)]
        token = getattr(self.tokenizer, "bos_token", None)
        if token:
            return self.tokenizer.encode(token, add_special_tokens=False)
        return []

    def _maybe_prepend_bos_to_chunk(self, chunk_ids: Sequence[int]) -> List[int]:
        ids = list(chunk_ids)
        if not self.config.chunk_bos:
            return ids
        bos = self._get_bos_token_ids()
        if not bos or ids[:len(bos)] == bos:
            return ids
        out = bos + ids
        size = int(self.config.chunk_size or 0)
        return out[:size] if size > 0 and len(out) > size else out  # a full chunk loses its last token (reference :904-908)

    @staticmethod
    def _window_query(query_ids: Sequence[int], window: int) -> List[int]:
        ids = list(query_ids)
        return ids[-window:] if window and window > 0 else ids

    @staticmethod
    def _range_positions(start: int, length: int) -> List[int]:
        return list(range(int(start), int(start) + int(length)))

    # RoPE position of the first token of a chunk / of the query window behind a chunk / of the final query, per position mode
    # (reference :922-948). One window of `chunk_size` positions is the unit: "reuse" puts every chunk in the same window right
    # behind the prefix, "continuous" stacks the selected chunks in selection order, "absolute" keeps a chunk where the full
    # context had it.
    def _window(self) -> int:
        return max(1, self.config.chunk_size)

    def _chunk_rope_start(self, prefix_len: int, chunk_order: int, chunk_index: int) -> int:
        mode = self.config.chunk_position_mode
        windows_before = {"reuse": 0, "continuous": chunk_order, "absolute": chunk_index}
        if mode not in windows_before:
            raise ValueError(f"Unsupported chunk_position_mode: {mode}")
        return prefix_len + windows_before[mode] * self._window()

    def _chunk_query_rope_start(self, prefix_len: int, chunk_start: int, chunk_len: int) -> int:
        mode = self.config.chunk_query_position_mode
        starts = {"after_reused_window": prefix_len + self._window(), "after_chunk": chunk_start + chunk_len}
        if mode not in starts:
            raise ValueError(f"Unsupported chunk_query_position_mode: {mode}")
        return starts[mode]

    def _final_query_rope_start(self, prefix_len: int, cache_positions: Sequence[int], selected_count: int) -> int:
        mode = self.config.query_position_mode
        if mode == "after_cache":
            return max(cache_positions, default=prefix_len - 1) + 1
        windows_before = {"after_reused_window": 1, "after_selected_chunks": selected_count}
        if mode not in windows_before:
            raise ValueError(f"Unsupported query_position_mode: {mode}")
        return prefix_len + windows_before[mode] * self._window()

    @staticmethod
    def _select_attention_layer_indices(total_layers: int, layer_window: int, layer_mode: str) -> List[int]:
        """Layers whose attention is scored: all of them, or a window of `layer_window` at either end (reference :1770-1780)."""
        every = list(range(max(0, total_layers)))
        if not every or layer_mode == "all" or layer_window <= 0:
            return every
        if layer_mode not in ("first", "last"):
            raise ValueError(f"Unsupported attention layer mode: {layer_mode}")
        width = min(max(1, int(layer_window)), total_layers)
        return every[:width] if layer_mode == "first" else every[-width:]

    @staticmethod
    def _mask_kind(mode: str) -> str:
        """"full" | "causal" | "query_to_chunk" (reference _attention_mask :982-1005)."""
        mode = (mode or "full").lower()
        if mode in {"full", "none"}:
            return "full"
        if mode in {"causal", "query_to_chunk"}:
            return mode
        raise ValueError(f"Unsupported attention mask mode: {mode}")

    def _mask_args(self, mode: str, *, rows_before_chunk: int, chunk_len: int, query_len: int) -> dict:
        """Keyword arguments of `_forward_packed` that realise a reference mask over the NEW rows [.. ‖ chunk ‖ query] of every
        packed sequence. "query_to_chunk" (reference _query_to_chunk_mask :963-980): everything is visible except that the
        chunk's rows do not see the query's keys — a dense bool mask with sequence-local indices, shared by the sequences."""
        kind = self._mask_kind(mode)
        if kind == "causal":
            return dict(causal=True)
        if kind == "full" or query_len <= 0 or chunk_len <= 0:
            return dict(causal=False)
        rows = rows_before_chunk + chunk_len + query_len
        visible = torch.ones((rows, rows), dtype=torch.bool, device=self.device)
        visible[rows_before_chunk:rows_before_chunk + chunk_len, rows_before_chunk + chunk_len:] = False
        return dict(causal=False, row_mask=visible)

    # ------------------------------------------------------------------------------------------------ model calls
    def _forward_packed(self, seqs_ids: Sequence[Sequence[int]], seqs_positions: Sequence[Sequence[int]], *, causal: bool,
                        cache: Optional[PagedCache] = None, ctx_len: int = 0, store_slots: Optional[Sequence[int]] = None,
                        logit_rows: Optional[Sequence[int]] = None, want_logits: bool = True, capture_layers=None,
                        ids_tensor: Optional[torch.Tensor] = None, store_after_attention: bool = False,
                        store_unrotated_k: bool = False, row_mask: Optional[torch.Tensor] = None):
        """One packed forward over several sequences; every sequence sees the first `ctx_len` tokens of `cache`. `row_mask`:
        bool [rows, rows] visibility among the new rows, the same for every sequence (all of one length then)."""
        m = self.model
        flat_pos = [p for seq in seqs_positions for p in seq]
        if ids_tensor is None:
            ids_tensor = m.ids_tensor([t for seq in seqs_ids for t in seq])
        lens = [len(seq) for seq in seqs_positions]
        cu = [0]
        for n in lens:
            cu.append(cu[-1] + n)
        kwargs = {}
        if cache is not None and ctx_len > 0:
            kwargs = dict(block_table=cache.table().expand(len(lens), -1).contiguous(),
                          seq_lens=m.i32([ctx_len + n for n in lens]), max_seq_len=ctx_len + max(lens))
        return m.forward(ids_tensor, torch.tensor(flat_pos, dtype=torch.long, device=m.device), cu_seqlens=m.i32(cu),
                         max_query_len=max(lens), slot_mapping=None if store_slots is None else m.i32(store_slots),
                         causal=causal, logit_rows=None if logit_rows is None else m.ids_tensor(logit_rows),
                         want_logits=want_logits, capture_qk_layers=capture_layers, store_after_attention=store_after_attention,
                         store_unrotated_k=store_unrotated_k, new_row_mask=row_mask, **kwargs)

    # ------------------------------------------------------------------------------------------------ draft
    def _draft_cache(self, past: Optional[PagedCache], extra_tokens: int) -> PagedCache:
        """The cache a draft works in: empty, or a PRIVATE copy of the given cache's pages (one copy launch over the K and V planes
        of all layers) with room for the query and the draft block behind it — the reference concatenates new tensors and
        leaves its caller's cache alone (:2614-2624); pages would otherwise be written past the caller's length."""
        if past is None or past.length <= 0:
            return PagedCache(self, extra_tokens)
        m = self.model
        cache = PagedCache(self, past.length + extra_tokens)
        try:
            n_pages = math.ceil(past.length / m.page_size)
            layers, pool_pages = int(m.kv_cache.shape[1]), int(m.kv_cache.shape[2])
            offsets = (torch.arange(2 * layers, dtype=torch.int32, device=m.device) * pool_pages).unsqueeze(1)
            pools = m.kv_cache.view(2 * layers * pool_pages, m.kv_cache.shape[3], m.kv_cache.shape[4], m.kv_cache.shape[5])
            src = (offsets + m.i32(past.page_ids[:n_pages]).unsqueeze(0)).reshape(-1)
            dst = (offsets + m.i32(cache.page_ids[:n_pages]).unsqueeze(0)).reshape(-1)
            ops.copy_pages(pools, src, pools, dst, n_lists=2 * layers, tokens_per_list=past.length)
            cache.length = past.length
            cache.positions = list(past.positions)
        except BaseException:
            cache.release()
            raise
        return cache

    @torch.inference_mode()
    def generate_partial_draft_rounds_from_cache(self, *, past_key_values: Optional[PagedCache], cache_positions: Sequence[int],
                                                 query_ids: Sequence[int], query_rope_start: int, max_new_tokens: int,
                                                 partial_rounds: int) -> Tuple[List[int], List[bool]]:
        """Draft `max_new_tokens` slots after the query: slot 0 from the last context logit, then `partial_rounds` rounds
        each confirming the single most confident masked slot (reference :2595-2676). Unfilled slots stay MASK."""
        draft_len = int(max_new_tokens)
        if draft_len <= 0:
            return [], []
        query_ids = list(query_ids)
        mask_id = self._mask_token_id()
        q_pos = self._range_positions(query_rope_start, len(query_ids))
        cache = self._draft_cache(past_key_values, len(query_ids) + draft_len)
        try:
            last_logit = None
            if query_ids:
                base = cache.length       # the given cache's tokens (a private copy of its pages): the query rows see them
                logits, _ = self._forward_packed([query_ids], [q_pos], causal=False, store_slots=cache.slots(base, len(query_ids)),
                                                 logit_rows=[len(query_ids) - 1], cache=cache if base else None, ctx_len=base)
                last_logit = logits[0]
                cache.length = base + len(query_ids)
            block_pos = self._range_positions(query_rope_start + len(query_ids), draft_len)
            block = torch.full((draft_len,), mask_id, dtype=torch.long, device=self.device)
            confirmed = torch.zeros(draft_len, dtype=torch.bool, device=self.device)
            if last_logit is not None:
                block[0] = self._first_block_token(last_logit, cache, block_pos)
            else:
                raise ValueError("draft needs at least one context token")
            confirmed[0] = True
            for _ in range(max(0, int(partial_rounds))):
                before = block.clone()
                logits, _ = self._forward_packed([[0] * draft_len], [block_pos], causal=False, cache=cache, ctx_len=cache.length,
                                                 ids_tensor=block)
                # only the top-1 slot is transferred in a draft round: a threshold above any probability
                if self._custom_sampling():
                    self._fill_most_confident(logits, block, last_logit, 1)
                else:
                    ops.unmask_step(logits, block, mask_token_id=mask_id, threshold=2.0, last_logit=last_logit,
                                    shift=self.arch.logit_shift)
                confirmed |= block != before
            return block.tolist(), confirmed.tolist()
        finally:
            cache.release()

    # ---- samplers off the fused path -----------------------------------------------------------------------------------
    def manual_seed(self, seed: int) -> None:
        """Seed the draws of the sampled paths (temperature > 0, alg_temp > 0)."""
        self.sampling_generator = torch.Generator(device=self.device)
        self.sampling_generator.manual_seed(int(seed))

    def _custom_sampling(self) -> bool:
        cfg = self.config
        return bool((cfg.temperature and cfg.temperature > 0) or cfg.top_p is not None or cfg.top_k is not None)

    def _slot_candidates(self, logits: torch.Tensor, block: torch.Tensor, last_logit: Optional[torch.Tensor], alg: str):
        """(is-MASK [n], confidence [masked], token [masked]) of one denoise forward under the configured sampler; `alg` picks the
        confidence (reference :2469-2493: max probability for origin / confidence_threshold, top-1 minus top-2 for topk_margin,
        negative entropy for anything else)."""
        cfg = self.config
        mask_index = block == self._mask_token_id()
        if self.arch.logit_shift:
            first = logits[:1] if last_logit is None else last_logit.reshape(1, -1)
            logits = torch.cat([first, logits[:-1]], dim=0)
        conf, tok = sample_tokens(logits[mask_index], temperature=float(cfg.temperature or 0.0), top_p=cfg.top_p, top_k=cfg.top_k,
                                  margin_confidence=alg == "topk_margin",
                                  neg_entropy=alg not in {"origin", "confidence_threshold", "topk_margin"}, generator=self.sampling_generator)
        return mask_index, conf, tok

    def _pick_first_token(self, last_logit: torch.Tensor) -> torch.Tensor:
        cfg = self.config
        return sample_tokens(last_logit.reshape(1, -1), temperature=float(cfg.temperature or 0.0), top_p=cfg.top_p, top_k=cfg.top_k,
                             generator=self.sampling_generator)[1][0]

    def _threshold_step_sampled(self, logits: torch.Tensor, block: torch.Tensor, last_logit: Optional[torch.Tensor]) -> int:
        """The confidence-threshold accept rule (reference :2414-2440) over `_slot_candidates`: the most confident MASK slot
        always, every other one whose confidence reaches the threshold. Returns the MASK slots left."""
        mask_index, conf, tok = self._slot_candidates(logits, block, last_logit, "confidence_threshold")
        n = int(conf.numel())
        if n == 0:
            return 0
        accept = conf >= float(self.config.threshold)
        accept[torch.argmax(conf)] = True
        slots = torch.nonzero(mask_index).reshape(-1)
        block[slots[accept]] = tok[accept]
        return n - int(accept.sum().item())

    def _fill_most_confident(self, logits: torch.Tensor, block: torch.Tensor, last_logit: Optional[torch.Tensor], count: int,
                             alg: str = "origin") -> int:
        """Fill `count` MASK slots of `block` (in place): the transfer rule of the fixed-step diffusion sampler and of the partial
        draft (reference :2548-2552, :2497-2510). With the default sampler (greedy, max-probability confidence, alg_temp 0)
        confidence and arg-max of every candidate slot come from the unmask kernel run on a scratch copy with a threshold no
        probability reaches, and the `count` most confident are taken; ties at the cut are as unspecified as torch.topk's in
        the reference. Otherwise the candidates come from `_slot_candidates` and, with alg_temp > 0, the slots are drawn
        without replacement from softmax(confidence / alg_temp). Returns slots filled."""
        if count <= 0:
            return 0
        cfg = self.config
        alg_temp = float(cfg.alg_temp or 0.0)
        if not self._custom_sampling() and alg in {"origin", "confidence_threshold"} and alg_temp == 0.0:
            scratch = block.clone()
            counts, conf, x0 = ops.unmask_step(logits, scratch, mask_token_id=self._mask_token_id(), threshold=2.0, last_logit=last_logit,
                                               shift=self.arch.logit_shift, return_details=True)
            count = min(int(count), int(counts[0].item()))
            if count <= 0:
                return 0
            idx = torch.topk(conf, count).indices
            block[idx] = x0[idx]
            return count
        mask_index, conf, tok = self._slot_candidates(logits, block, last_logit, alg)
        count = min(int(count), int(conf.numel()))
        if count <= 0:
            return 0
        if alg_temp == 0.0:
            pick = torch.topk(conf, count).indices
        else:
            pick = torch.multinomial(torch.softmax(conf.float() / alg_temp, dim=-1), count, generator=self.sampling_generator)
        slots = torch.nonzero(mask_index).reshape(-1)
        block[slots[pick]] = tok[pick]
        return count

    @torch.inference_mode()
    def generate_partial_draft_from_cache(self, *, past_key_values: Optional[PagedCache], cache_positions: Sequence[int], query_ids,
                                          query_rope_start: int, max_new_tokens: int, partial_steps: int) -> Tuple[List[int], int]:
        """Draft that stops once `partial_steps` slots are filled: slot 0 from the last context logit, then forwards that
        each fill as many of the most confident slots as are still wanted (reference :2512-2593). Returns (ids, filled)."""
        draft_len = int(max_new_tokens)
        if draft_len <= 0:
            return [], 0
        query_ids = list(query_ids)
        if not query_ids:
            raise ValueError("draft needs at least one context token")
        mask_id = self._mask_token_id()
        cache = self._draft_cache(past_key_values, len(query_ids) + draft_len)
        try:
            q_pos = self._range_positions(query_rope_start, len(query_ids))
            base = cache.length
            logits, _ = self._forward_packed([query_ids], [q_pos], causal=False, store_slots=cache.slots(base, len(query_ids)),
                                             logit_rows=[len(query_ids) - 1], cache=cache if base else None, ctx_len=base)
            last_logit = logits[0]
            cache.length = base + len(query_ids)
            block_pos = self._range_positions(query_rope_start + len(query_ids), draft_len)
            block = torch.full((draft_len,), mask_id, dtype=torch.long, device=self.device)
            target = min(draft_len, max(0, int(partial_steps)))
            filled = 0
            if target > 0:
                block[0] = self._first_block_token(last_logit, cache, block_pos)
                filled = 1
            while filled < target and bool((block == mask_id).any()):
                logits, _ = self._forward_packed([[0] * draft_len], [block_pos], causal=False, cache=cache, ctx_len=cache.length,
                                                 ids_tensor=block)
                done = self._fill_most_confident(logits, block, last_logit, target - filled)
                if done <= 0:
                    break
                filled += done
            return block.tolist(), filled
        finally:
            cache.release()

    def _first_block_token(self, last_logit: torch.Tensor, cache: Optional[PagedCache] = None, block_pos: Optional[Sequence[int]] = None) -> torch.Tensor:
        """First token of a block (reference _initialize_fastdllm_suffix_cache :2368-2397): Dream reads it from the last context
        logit; an un-shifted architecture (LLaDA) from the first MASK slot's own row of a forward of the all-MASK block over
        the cached context."""
        if not self.arch.logit_shift:
            if cache is None or block_pos is None:
                raise ValueError("the un-shifted read-out needs the cached context to initialise a block")
            n = len(block_pos)
            logits, _ = self._forward_packed([[self._mask_token_id()] * n], [list(block_pos)], causal=False, cache=cache, ctx_len=cache.length,
                                             logit_rows=[0])
            last_logit = logits[0]
        if self._custom_sampling():
            return self._pick_first_token(last_logit)
        return torch.argmax(last_logit)   # softmax is monotone: the arg-max of the logit

    def _selection_query_ids_with_score_target(self, prefix_ids, scoring_query_ids):
        selection = list(scoring_query_ids)
        score_token_mask: Optional[List[bool]] = None
        cfg = self.config
        if cfg.score_mode == "draft_self_information" and cfg.score_draft_tokens > 0:
            draft_query = list(prefix_ids) + list(scoring_query_ids)
            if cfg.score_draft_partial_rounds is not None:
                draft_ids, draft_mask = self.generate_partial_draft_rounds_from_cache(
                    past_key_values=None, cache_positions=[], query_ids=draft_query, query_rope_start=0,
                    max_new_tokens=int(cfg.score_draft_tokens), partial_rounds=int(cfg.score_draft_partial_rounds))
                if cfg.score_draft_score_all_slots:
                    score_token_mask = [True] * len(scoring_query_ids) + [True] * len(draft_ids)
                else:
                    score_token_mask = [True] * len(scoring_query_ids) + list(draft_mask)
            elif cfg.score_draft_partial_steps is not None:
                draft_ids, _ = self.generate_partial_draft_from_cache(
                    past_key_values=None, cache_positions=[], query_ids=draft_query, query_rope_start=0,
                    max_new_tokens=int(cfg.score_draft_tokens), partial_steps=int(cfg.score_draft_partial_steps))
                mask_id = self._mask_token_id()
                score_token_mask = [True] * len(scoring_query_ids) + [t != mask_id for t in draft_ids]
            else:
                # the dataclass default (reference :1828-1837): a complete draft, every query + draft position is a label
                draft_ids = self.generate_from_cache(
                    past_key_values=None, cache_positions=[], query_ids=draft_query, query_rope_start=0,
                    max_new_tokens=int(cfg.score_draft_tokens), diffusion_steps=int(cfg.score_draft_steps or 1),
                    force_diffusion=bool(cfg.score_draft_fixed_steps))
            selection = list(scoring_query_ids) + draft_ids
        return selection, None, score_token_mask

    # ------------------------------------------------------------------------------------------------ scoring + ranking
    @torch.inference_mode()
    def score_chunks_self_information_batched(self, prefix_ids, candidate_chunks, query_ids, score_token_count=None,
                                              score_token_mask=None) -> Dict[int, float]:
        """mean log p(label | prefix, chunk, earlier query) per chunk (reference :1314-1423): causal forward of
        [prefix‖chunk‖query‖draft] rows batched by chunk length, LM head on the label rows only, fused fp32 tail."""
        cfg = self.config
        if score_token_count is None and score_token_mask is None:
            query_ids = self._window_query(query_ids, cfg.score_query_window)
        query_ids, prefix_ids = list(query_ids), list(prefix_ids)
        if not query_ids:
            return {i: float("-inf") for i in range(len(candidate_chunks))}
        p_len, q_len = len(prefix_ids), len(query_ids)
        scores: Dict[int, float] = {}
        groups: Dict[int, List[Tuple[int, List[int]]]] = {}
        for idx, chunk in enumerate(candidate_chunks):
            chunk = list(chunk)
            if not chunk:
                scores[idx] = float("-inf")
            else:
                groups.setdefault(len(chunk), []).append((idx, chunk))
        batch_size = max(1, int(cfg.score_batch_size or 1))
        for c_len, group in groups.items():
            if score_token_mask is not None:
                if len(score_token_mask) != q_len:
                    scores.update({idx: float("-inf") for idx, _ in group})
                    continue
                local = [i for i, keep in enumerate(score_token_mask) if keep]
            elif score_token_count is None:
                window = min(q_len, cfg.score_query_window or q_len)
                local = list(range(q_len - window, q_len))
            else:
                local = list(range(min(q_len, max(0, int(score_token_count)))))    # the FIRST tokens of the query
            if not local:
                scores.update({idx: float("-inf") for idx, _ in group})
                continue
            label_pos = [p_len + c_len + i for i in local]
            if min(label_pos) <= 0:
                scores.update({idx: float("-inf") for idx, _ in group})
                continue
            labels = self.model.ids_tensor([query_ids[i] for i in local])
            row_len = p_len + c_len + q_len
            positions = list(range(row_len))
            mask_args = self._mask_args(cfg.score_attention_mask, rows_before_chunk=p_len, chunk_len=c_len, query_len=q_len)
            if self.model_backend == "llada" and not cfg.score_llada_shift_logits:
                for idx, chunk in group:
                    scores[idx] = self._leave_one_out_score(prefix_ids + chunk + query_ids, label_pos, [query_ids[i] for i in local], mask_args)
                continue
            for off in range(0, len(group), batch_size):
                batch = group[off:off + batch_size]
                rows = [prefix_ids + chunk + query_ids for _, chunk in batch]
                logit_rows = [b * row_len + (p - 1) for b in range(len(batch)) for p in label_pos]  # label p reads logits[p-1]
                logits, _ = self._forward_packed(rows, [positions] * len(batch), logit_rows=logit_rows, **mask_args)
                vals = ops.self_information_scores(logits, labels, len(batch)).tolist()
                for (idx, _), v in zip(batch, vals):
                    scores[idx] = v if math.isfinite(v) else float("-inf")
        return scores

    def _leave_one_out_score(self, joint_ids: Sequence[int], label_positions: Sequence[int], label_ids: Sequence[int], mask_args: dict) -> float:
        """Masked-diffusion self-information (reference _llada_leave_one_out_score :1166-1201): one copy of the row per label with
        that label replaced by MASK, `llada_score_batch_size` copies per packed forward, the label's log-probability read at
        its OWN row; the mean over the labels."""
        if not label_positions:
            return float("-inf")
        mask_id = self._mask_token_id()
        batch_size = max(1, int(self.config.llada_score_batch_size or 1))
        row_len = len(joint_ids)
        positions = list(range(row_len))
        base = self.model.ids_tensor(list(joint_ids))
        total, count = 0.0, 0
        for off in range(0, len(label_positions), batch_size):
            pos = [int(p) for p in label_positions[off:off + batch_size]]
            ids = base.repeat(len(pos))
            rows = [b * row_len + p for b, p in enumerate(pos)]
            ids[self.model.ids_tensor(rows)] = mask_id
            logits, _ = self._forward_packed([joint_ids] * len(pos), [positions] * len(pos), ids_tensor=ids, logit_rows=rows, **mask_args)
            labels = self.model.ids_tensor([int(t) for t in label_ids[off:off + batch_size]])
            _, nll = ops.self_information_scores(logits, labels, 1, return_nll=True)      # row i against label i: -log p
            total -= float(nll.sum().item())
            count += len(pos)
        value = total / max(1, count)
        return value if math.isfinite(value) else float("-inf")

    def score_chunk_self_information(self, prefix_ids, chunk_ids, query_ids, score_token_count=None, score_token_mask=None) -> float:
        """One chunk's score (reference :1258-1312): the batched scorer on a batch of one."""
        return self.score_chunks_self_information_batched(prefix_ids, [list(chunk_ids)], query_ids, score_token_count=score_token_count,
                                                          score_token_mask=score_token_mask).get(0, float("-inf"))

    @torch.inference_mode()
    def score_chunk_self_information_joint_chunks(self, prefix_ids, candidate_chunks, target_index: int, query_ids,
                                                  score_token_count=None, score_token_mask=None) -> float:
        """Score chunk `target_index` with every other chunk in front of it in the same forward: rows
        [prefix ‖ other chunks in order ‖ target chunk ‖ query], labels as in the single-chunk score (reference :1425-1505)."""
        cfg = self.config
        if score_token_count is None and score_token_mask is None:
            query_ids = self._window_query(query_ids, cfg.score_query_window)
        query_ids, prefix_ids = list(query_ids), list(prefix_ids)
        if not candidate_chunks or not query_ids or not 0 <= target_index < len(candidate_chunks):
            return float("-inf")
        target = list(candidate_chunks[target_index])
        if not target:
            return float("-inf")
        context = [t for i, c in enumerate(candidate_chunks) if i != target_index for t in c] + target
        joint = prefix_ids + context + query_ids
        p_len, c_len, q_len = len(prefix_ids), len(context), len(query_ids)
        if score_token_mask is not None:
            if len(score_token_mask) != q_len:
                return float("-inf")
            local = [i for i, keep in enumerate(score_token_mask) if keep]
        elif score_token_count is None:
            window = min(q_len, cfg.score_query_window or q_len)
            local = list(range(q_len - window, q_len))
        else:
            local = list(range(min(q_len, max(0, int(score_token_count)))))
        if not local:
            return float("-inf")
        label_pos = [p_len + c_len + i for i in local]
        if min(label_pos) <= 0:
            return float("-inf")
        mask_args = self._mask_args(cfg.score_attention_mask, rows_before_chunk=p_len, chunk_len=c_len, query_len=q_len)
        if self.model_backend == "llada" and not cfg.score_llada_shift_logits:
            return self._leave_one_out_score(joint, label_pos, [query_ids[i] for i in local], mask_args)
        logits, _ = self._forward_packed([joint], [list(range(len(joint)))], logit_rows=[p - 1 for p in label_pos], **mask_args)
        value = float(ops.self_information_scores(logits, self.model.ids_tensor([query_ids[i] for i in local]), 1)[0].item())
        return value if math.isfinite(value) else float("-inf")

    @torch.inference_mode()
    def score_chunk_next_block_logits(self, prefix_ids, chunk_ids, query_ids) -> float:
        """Mean fp32 max-probability of `score_draft_tokens` MASK slots appended to [prefix ‖ chunk ‖ query], one bidirectional
        forward (reference :1507-1529; Dream reads slot j at the logit row before it)."""
        cfg = self.config
        draft_len = max(1, int(cfg.score_draft_tokens or cfg.block_length or 1))
        if not chunk_ids or not query_ids:
            return float("-inf")
        joint = list(prefix_ids) + list(chunk_ids) + list(query_ids) + [self._mask_token_id()] * draft_len
        first = len(joint) - draft_len
        shift = 1 if self.arch.logit_shift else 0
        rows = [max(0, first + j - shift) for j in range(draft_len)]
        logits, _ = self._forward_packed([joint], [list(range(len(joint)))], causal=False, logit_rows=rows)
        return float(torch.softmax(logits.float(), dim=-1).max(dim=-1).values.mean().item())

    def select_chunks(self, prefix_ids, candidate_chunks, scoring_query_ids):
        """(selected ascending, scores, selection query ids, label mask) — reference :1857-1953."""
        cfg = self.config
        if not candidate_chunks:
            return [], {}, list(scoring_query_ids), None
        selection, count, mask = self._selection_query_ids_with_score_target(prefix_ids, scoring_query_ids)
        if cfg.score_mode == "none" or not selection:
            selected = list(range(len(candidate_chunks)))
            if cfg.topk_chunks > 0:
                selected = selected[:cfg.topk_chunks]
            return selected, {}, selection, mask
        scores: Dict[int, float] = {}
        if cfg.score_mode in {"self_information", "draft_self_information"}:
            if cfg.score_context_mode == "single_chunk":
                # the batched and the one-by-one scorer of the reference compute the same value per chunk; batch size 1 packs one
                scores = self.score_chunks_self_information_batched(prefix_ids, candidate_chunks, selection, score_token_count=count,
                                                                    score_token_mask=mask)
            elif cfg.score_context_mode == "joint_chunks_target_last":
                for idx in range(len(candidate_chunks)):
                    scores[idx] = self.score_chunk_self_information_joint_chunks(prefix_ids, candidate_chunks, idx, selection,
                                                                                 score_token_count=count, score_token_mask=mask)
            else:
                raise ValueError(f"Unsupported score_context_mode: {cfg.score_context_mode}")
        elif cfg.score_mode == "per_chunk_draft_self_information":
            for idx, chunk in enumerate(candidate_chunks):
                per_chunk_query = list(scoring_query_ids)
                if cfg.score_draft_tokens > 0:
                    per_chunk_query += self.generate_from_cache(
                        past_key_values=None, cache_positions=[], query_ids=list(prefix_ids) + list(chunk) + list(scoring_query_ids),
                        query_rope_start=0, max_new_tokens=int(cfg.score_draft_tokens), diffusion_steps=int(cfg.score_draft_steps or 1),
                        force_diffusion=bool(cfg.score_draft_fixed_steps))
                scores[idx] = self.score_chunk_self_information(prefix_ids, chunk, per_chunk_query)
        elif cfg.score_mode == "next_block_logits":
            for idx, chunk in enumerate(candidate_chunks):
                scores[idx] = self.score_chunk_next_block_logits(prefix_ids, chunk, scoring_query_ids)
        elif cfg.score_mode == "attention":
            for idx, chunk in enumerate(candidate_chunks):
                token_scores = self.query_attention_token_scores(
                    prefix_ids, chunk, selection, query_window=cfg.attention_query_window, layer_window=cfg.attention_score_layers,
                    layer_mode="last", reduce_mode=cfg.token_score_reduce, pooling=cfg.token_score_pooling,
                    pool_kernel=cfg.token_score_pool_kernel, head_reduce=cfg.token_score_head_reduce, layer_reduce=cfg.token_score_layer_reduce)
                scores[idx] = float(token_scores.mean().item()) if token_scores.numel() else float("-inf")
        else:
            raise ValueError(f"Unsupported score_mode: {cfg.score_mode}")
        scores = {i: (v if math.isfinite(v) else float("-inf")) for i, v in scores.items()}
        dense = torch.tensor([scores.get(i, float("-inf")) for i in range(len(candidate_chunks))], dtype=torch.float32,
                             device=self.device)
        sel, cnt = ops.topk_chunks(dense, int(cfg.topk_chunks), bool(cfg.keep_first_chunk))
        selected = sel[: int(cnt.item())].tolist()
        return selected, scores, selection, mask

    def _token_eviction_query_ids(self, scoring_query_ids, selection_query_ids, score_token_mask):
        if not self.config.token_score_use_generated:
            return list(scoring_query_ids)
        if score_token_mask is not None and len(score_token_mask) == len(selection_query_ids):
            return [int(t) for t, keep in zip(selection_query_ids, score_token_mask) if keep]
        return list(selection_query_ids)

    # ------------------------------------------------------------------------------------------------ token eviction
    @torch.inference_mode()
    def _chunk_head_scores(self, prefix_ids, chunk_ids, query_ids, *, query_window=None, layer_window=None, layer_mode=None,
                           reduce_mode=None) -> Optional[Tuple[torch.Tensor, List[int]]]:
        """fp32 [selected layers, Hq, chunk_len] attention mass between the last `query_window` query tokens and the chunk's
        tokens (reference query_attention_token_scores :1531-1637 / _chunk_attention_head_scores :1639-1667). Direction
        query→chunk comes from the fused scorer on the layer's rotated (q, k); chunk→query (and their sum, "bidirectional")
        needs the chunk rows' own softmax and is computed from the same (q, k) with device-side matrix products."""
        cfg = self.config
        query_ids = self._window_query(query_ids, cfg.token_score_query_window if query_window is None else query_window)
        if not chunk_ids or not query_ids:
            return None
        prefix = list(prefix_ids) if cfg.token_score_include_prefix else []
        joint = prefix + list(chunk_ids) + list(query_ids)
        layers = self._select_attention_layer_indices(self.arch.num_hidden_layers,
                                                      cfg.token_score_layers if layer_window is None else layer_window,
                                                      cfg.token_score_layer_mode if layer_mode is None else layer_mode)
        if not layers:
            return None
        p_len, c_len, q_len = len(prefix), len(chunk_ids), len(query_ids)
        reduce_mode = cfg.token_score_reduce if reduce_mode is None else reduce_mode
        mask_args = self._mask_args(cfg.token_attention_mask, rows_before_chunk=p_len, chunk_len=c_len, query_len=q_len)
        _, captured = self._forward_packed([joint], [list(range(len(joint)))], want_logits=False, capture_layers=layers, **mask_args)
        direction = cfg.token_score_direction
        per_layer = []
        for l in layers:
            q, k = captured[l]
            parts = []
            if direction in {"query_to_chunk", "bidirectional"}:
                parts.append(ops.query_to_chunk_attention_scores(q, k, prefix_len=p_len, chunk_len=c_len, query_len=q_len, scale=self.model.scale,
                                                                 reduce_mode=reduce_mode, attention_mask=cfg.token_attention_mask))
            if direction in {"chunk_to_query", "bidirectional"}:
                parts.append(self._chunk_to_query_mass(q, k, p_len, c_len, q_len, reduce_mode, mask_args))
            per_layer.append(parts[0] if len(parts) == 1 else parts[0] + parts[1])
        return torch.stack(per_layer, dim=0).contiguous(), layers

    @torch.inference_mode()
    def _chunk_head_scores_packed(self, prefix_ids, chunks: Sequence[Sequence[int]], query_ids):
        """`_chunk_head_scores` of several chunks of ONE length in one packed forward (the chunks are independent sequences: same
        arithmetic per chunk, one pass over the weights for all of them). Returns one (head scores, layers) pair per chunk,
        or None where `_chunk_head_scores` would return None."""
        cfg = self.config
        window = self._window_query(query_ids, cfg.token_score_query_window)
        layers = self._select_attention_layer_indices(self.arch.num_hidden_layers, cfg.token_score_layers, cfg.token_score_layer_mode)
        if not window or not layers or not chunks or not chunks[0]:
            return [None] * len(chunks)
        prefix = list(prefix_ids) if cfg.token_score_include_prefix else []
        p_len, c_len, q_len = len(prefix), len(chunks[0]), len(window)
        row_len = p_len + c_len + q_len
        mask_args = self._mask_args(cfg.token_attention_mask, rows_before_chunk=p_len, chunk_len=c_len, query_len=q_len)
        _, captured = self._forward_packed([prefix + list(c) + window for c in chunks], [list(range(row_len))] * len(chunks), want_logits=False,
                                           capture_layers=layers, **mask_args)
        out = []
        for b in range(len(chunks)):
            rows = slice(b * row_len, (b + 1) * row_len)
            per_layer = [ops.query_to_chunk_attention_scores(captured[l][0][rows], captured[l][1][rows], prefix_len=p_len, chunk_len=c_len,
                                                             query_len=q_len, scale=self.model.scale, reduce_mode=cfg.token_score_reduce,
                                                             attention_mask=cfg.token_attention_mask) for l in layers]
            out.append((torch.stack(per_layer, dim=0).contiguous(), layers))
        return out

    def _chunk_to_query_mass(self, q: torch.Tensor, k: torch.Tensor, p_len: int, c_len: int, q_len: int, reduce_mode: str, mask_args: dict):
        """fp32 [Hq, chunk_len]: attention probability that each chunk row puts on the query's keys, summed (or averaged) over
        those keys, under the forward's own mask. Zero under the causal and query_to_chunk masks (chunk rows do not see the query)."""
        hq, hkv = self.arch.num_attention_heads, self.arch.num_key_value_heads
        if mask_args.get("causal") or mask_args.get("row_mask") is not None:
            return torch.zeros((hq, c_len), dtype=torch.float32, device=self.device)
        rows = q[p_len:p_len + c_len].float().transpose(0, 1)                              # [Hq, C, D]
        keys = k.float().transpose(0, 1).repeat_interleave(hq // hkv, dim=0)               # [Hq, L, D]
        prob = torch.softmax(torch.matmul(rows, keys.transpose(1, 2)) * self.model.scale, dim=-1)
        part = prob[:, :, p_len + c_len:p_len + c_len + q_len]
        return part.mean(dim=2) if reduce_mode == "mean" else part.sum(dim=2)

    @staticmethod
    def _pool_head_scores(head_scores: torch.Tensor, pooling: str, pool_kernel: int) -> torch.Tensor:
        """avg / max pooling along the chunk axis with stride 1 and half-kernel zero / -inf padding (reference :1607-1617)."""
        if pooling == "none" or head_scores.shape[-1] == 0:
            return head_scores
        kernel = max(1, min(int(pool_kernel), head_scores.shape[-1]))
        flat = head_scores.reshape(-1, 1, head_scores.shape[-1])
        if pooling == "avgpool":
            flat = torch.nn.functional.avg_pool1d(flat, kernel_size=kernel, padding=kernel // 2, stride=1)
        elif pooling == "maxpool":
            flat = torch.nn.functional.max_pool1d(flat, kernel_size=kernel, padding=kernel // 2, stride=1)
        else:
            raise ValueError(f"Unsupported token_score_pooling: {pooling}")
        return flat[..., :head_scores.shape[-1]].reshape(head_scores.shape)

    @torch.inference_mode()
    def query_attention_token_scores(self, prefix_ids, chunk_ids, query_ids, *, query_window: int, layer_window: int, layer_mode: str,
                                     reduce_mode: str, pooling: Optional[str] = None, pool_kernel: Optional[int] = None,
                                     head_reduce: Optional[str] = None, layer_reduce: Optional[str] = None) -> torch.Tensor:
        """fp32 [chunk_len] token scores: per selected layer pool each head's scores along the chunk, reduce over heads, then
        over layers (reference :1531-1637). Empty tensor when nothing can be scored."""
        cfg = self.config
        scored = self._chunk_head_scores(prefix_ids, chunk_ids, query_ids, query_window=query_window, layer_window=layer_window,
                                         layer_mode=layer_mode, reduce_mode=reduce_mode)
        if scored is None:
            return torch.empty(0, device=self.device)
        pooling = (pooling or cfg.token_score_pooling or "none").lower()
        head_reduce = (head_reduce or cfg.token_score_head_reduce or "sum").lower()
        layer_reduce = (layer_reduce or cfg.token_score_layer_reduce or "mean").lower()
        pooled = self._pool_head_scores(scored[0], pooling, int(pool_kernel or cfg.token_score_pool_kernel or 1))
        if head_reduce == "mean":
            per_layer = pooled.mean(dim=1)
        elif head_reduce == "sum":
            per_layer = pooled.sum(dim=1)
        elif head_reduce == "max":
            per_layer = pooled.max(dim=1).values
        else:
            raise ValueError(f"Unsupported token_score_head_reduce: {head_reduce}")
        if layer_reduce == "mean":
            return per_layer.mean(dim=0)
        if layer_reduce == "sum":
            return per_layer.sum(dim=0)
        if layer_reduce == "max":
            return per_layer.max(dim=0).values
        raise ValueError(f"Unsupported token_score_layer_reduce: {layer_reduce}")

    def _fused_reductions(self) -> Optional[int]:
        """The pool kernel width when the configured reductions are the ones the fused eviction kernel computes (max-pooling or
        none, heads summed, layers averaged); None when they have to be applied with tensor ops first."""
        cfg = self.config
        pooling = (cfg.token_score_pooling or "none").lower()
        if pooling not in {"none", "maxpool", "avgpool"}:
            raise ValueError(f"Unsupported token_score_pooling: {pooling}")
        if pooling == "avgpool" or (cfg.token_score_head_reduce or "sum").lower() != "sum" \
                or (cfg.token_score_layer_reduce or "mean").lower() != "mean":
            return None
        return 1 if pooling == "none" else int(cfg.token_score_pool_kernel or 1)

    def _keep_positions_for_chunk(self, prefix_ids, chunk_ids, query_ids, scored=_NOT_SCORED) -> List[int]:
        """Kept positions of one chunk (reference :1955-1995). `scored`: the chunk's head scores when the caller already ran the
        scoring forward for several chunks at once (`_chunk_head_scores_packed`)."""
        cfg = self.config
        capacity, chunk_len = int(cfg.token_capacity or 0), len(chunk_ids)
        if capacity <= 0 or chunk_len <= capacity:
            return list(range(chunk_len))
        pool_kernel = self._fused_reductions()
        force_bos = bool(cfg.force_keep_chunk_bos and cfg.chunk_bos)
        if pool_kernel is not None:
            if scored is _NOT_SCORED:
                scored = self._chunk_head_scores(prefix_ids, chunk_ids, query_ids)
            head_scores, n_heads = (None, 0) if scored is None else (scored[0], self.arch.num_key_value_heads)
        else:
            # reductions the fused kernel does not compute: reduce with tensor ops, then let the kernel rank one "head" of one "layer"
            token_scores = self.query_attention_token_scores(
                prefix_ids, chunk_ids, query_ids, query_window=cfg.token_score_query_window, layer_window=cfg.token_score_layers,
                layer_mode=cfg.token_score_layer_mode, reduce_mode=cfg.token_score_reduce)
            head_scores, n_heads, pool_kernel = (None, 0, 1) if token_scores.numel() != chunk_len else (token_scores.reshape(1, 1, -1).contiguous(), 1, 1)
        if head_scores is None:
            head = capacity // 2
            keep = sorted(set(list(range(head)) + list(range(chunk_len - (capacity - head), chunk_len))))
        else:
            keep = ops.evict_select(head_scores, num_kv_heads=n_heads, keep_count=min(max(1, capacity), chunk_len),
                                    pool_kernel=pool_kernel, per_head=False, force_keep_first=force_bos,
                                    keep_high=cfg.token_score_keep == "high")[0].tolist()
        if force_bos and chunk_len > 0:
            keep = sorted(set([0] + keep))
            if len(keep) > capacity:
                keep = sorted([0] + [i for i in keep if i != 0][-max(0, capacity - 1):])
        return keep

    def _keep_positions_per_layer_per_head_for_chunk(self, prefix_ids, chunk_ids, query_ids) -> List[torch.Tensor]:
        cfg = self.config
        capacity, chunk_len = int(cfg.token_capacity or 0), len(chunk_ids)
        n_layers, hkv = self.arch.num_hidden_layers, self.arch.num_key_value_heads
        if chunk_len <= 0:
            return []
        if capacity <= 0 or chunk_len <= capacity:
            base = torch.arange(chunk_len, device=self.device, dtype=torch.long)
            return [base.unsqueeze(0).expand(hkv, -1).clone() for _ in range(n_layers)]
        pool_kernel = self._fused_reductions()
        keep_count = min(capacity, chunk_len)
        scored = self._chunk_head_scores(prefix_ids, chunk_ids, query_ids)
        pooling = (cfg.token_score_pooling or "none").lower()
        if scored is not None and pooling == "avgpool":
            # per-head lists only pool and average the heads of a KV group (reference :1741-1760): pool here, group in the kernel
            scored = (self._pool_head_scores(scored[0], pooling, int(cfg.token_score_pool_kernel or 1)).contiguous(), scored[1])
            pool_kernel = 1
        elif pool_kernel is None:
            pool_kernel = 1 if pooling == "none" else int(cfg.token_score_pool_kernel or 1)
        if scored is None:
            head = keep_count // 2
            fb = torch.tensor(sorted(set(list(range(head)) + list(range(chunk_len - (keep_count - head), chunk_len))))[:keep_count],
                              device=self.device, dtype=torch.long)
            return [fb.unsqueeze(0).expand(hkv, -1).clone() for _ in range(n_layers)]
        head_scores, layers = scored
        keep = ops.evict_select(head_scores, num_kv_heads=hkv, keep_count=keep_count, pool_kernel=pool_kernel, per_head=True,
                                force_keep_first=bool(cfg.force_keep_chunk_bos and cfg.chunk_bos), keep_high=cfg.token_score_keep == "high")
        by_layer: List[Optional[torch.Tensor]] = [None] * n_layers
        for i, l in enumerate(layers):
            by_layer[l] = keep[i]
        fallback = keep[0]
        return [k if k is not None else fallback.clone() for k in by_layer]

    # ------------------------------------------------------------------------------------------------ block denoising
    def _denoise_blocks(self, cache: PagedCache, *, suffix_pos_start: int, last_logit: torch.Tensor,
                        first_token: Optional[torch.Tensor], tail_in_cache: int, max_new: int,
                        fixed_steps_per_block: Optional[int] = None, confidence_alg: Optional[str] = None) -> List[int]:
        """Fast-dLLM dual-cache block loop over the paged cache (reference :2932-2998, :2399-2441): `model.denoise_blocks`
        with this runtime's settings — softmax in the model dtype, as the eval class computes it."""
        if self.config.generation_position_mode != "after_query":
            raise ValueError(f"Unsupported generation_position_mode: {self.config.generation_position_mode}")
        alg = confidence_alg or self.config.alg
        sampled = self._custom_sampling()
        return denoise_blocks(self.model, cache, suffix_pos_start=suffix_pos_start, last_logit=last_logit, first_token=first_token,
                              tail_in_cache=tail_in_cache, max_new=max_new, block_length=self.block_length, mask_id=self._mask_token_id(),
                              threshold=float(self.config.threshold), softmax_dtype=None, use_graph=bool(self.config.decode_cuda_graph),
                              fixed_steps_per_block=fixed_steps_per_block,
                              fill_most_confident=lambda lg, blk, last, count: self._fill_most_confident(lg, blk, last, count, alg=alg),
                              pick_first_token=self._pick_first_token if sampled else None,
                              threshold_step=self._threshold_step_sampled if sampled else None)

    # ------------------------------------------------------------------------------------------------ chunk-local caches
    def _prefill_one_chunk(self, cache: "PagedCache", dst: int, prefix_ids, chunk, order: int, ci: int, evict_q, window_q):
        """Forward one selected chunk (with the query window behind it in chunk_query mode) against the prefix KV already in
        `cache` and leave its KEPT rows at cache tokens [dst, dst + kept). Returns (kept, kept positions, union of kept chunk
        indices, rope start). `order` is the chunk's rank among the selected ones, `ci` its index among the candidates."""
        cfg = self.config
        p_len = len(prefix_ids)
        per_head = cfg.token_eviction_granularity == "per_head"
        c_start = self._chunk_rope_start(p_len, order, ci)
        c_pos = self._range_positions(c_start, len(chunk))
        if per_head:
            keep_ph = self._keep_positions_per_layer_per_head_for_chunk(prefix_ids, chunk, evict_q)
            keep_union = sorted({int(v) for k in keep_ph for v in k.reshape(-1).tolist()}) if keep_ph else []
            kept = int(keep_ph[0].shape[1]) if keep_ph else len(chunk)
        else:
            keep_ph = None
            keep_union = self._keep_positions_for_chunk(prefix_ids, chunk, evict_q)
            kept = len(keep_union)
        rows_ids, rows_pos = chunk, c_pos
        if cfg.cache_build_mode == "chunk_query":
            tq_start = self._chunk_query_rope_start(p_len, c_start, len(chunk))
            rows_ids = chunk + window_q
            rows_pos = c_pos + self._range_positions(tq_start, len(window_q))
            # the prefix is cached context (always visible); the mask applies among the new rows [chunk ‖ query window]
            mask_args = self._mask_args(cfg.token_attention_mask, rows_before_chunk=0, chunk_len=len(chunk), query_len=len(window_q))
        else:
            mask_args = dict(causal=False)
        if per_head and keep_ph and kept < len(chunk):
            # all chunk rows go to a staging area behind the destination, K un-rotated; a per-head compaction moves
            # the kept ones; then kept row j of EVERY head is rotated to the j-th chunk position, as the reference's
            # model does when it rotates cached keys at read time with the compacted position list (:2284-2288)
            stage = dst + kept
            slots = cache.slots(stage, len(chunk)) + [-1] * (len(rows_ids) - len(chunk))
            self._forward_packed([rows_ids], [rows_pos], cache=cache if p_len else None, ctx_len=p_len,
                                 store_slots=slots, want_logits=False, store_unrotated_k=True, **mask_args)
            for layer in range(self.arch.num_hidden_layers):
                for kv in self.model.layer_cache(layer):
                    ops.compact_pages_per_head(kv, cache.page_ids, cache.page_ids, keep_ph[layer] + stage,
                                               src_tokens=stage + len(chunk), dst_start=dst)
            kept_pos = c_pos[:kept]
            self.model.rope_rows(cache.page_ids, dst, kept_pos)
        else:
            keep_set = set(keep_union)
            next_slot = iter(cache.slots(dst, kept))
            slots = [next(next_slot) if i in keep_set else -1 for i in range(len(chunk))] + [-1] * (len(rows_ids) - len(chunk))
            self._forward_packed([rows_ids], [rows_pos], cache=cache if p_len else None, ctx_len=p_len,
                                 store_slots=slots, want_logits=False, **mask_args)
            kept_pos = [c_pos[i] for i in keep_union]
        return kept, kept_pos, keep_union, c_start

    def _prefill_chunks_packed(self, cache: "PagedCache", dst: int, prefix_ids, items, evict_q, window_q):
        """`_prefill_one_chunk` for all selected chunks at once when eviction is global: the chunks are independent sequences
        (each attends the prefix KV and itself), so the token-scoring forwards of same-length chunks are ONE packed forward and so
        are their prefill forwards — one pass over the weights instead of one per chunk, and row counts at which the GEMM runs
        wide tiles. `items`: (order, chunk index, chunk ids) in cache order. Returns one (kept, kept positions, kept indices, rope
        start) per item with the kept rows laid out consecutively from cache token `dst`, or None when the per-chunk path has to
        run (per-head eviction, reductions or score directions the packed scorer does not cover, a single chunk)."""
        cfg = self.config
        if cfg.token_eviction_granularity == "per_head" or len(items) < 2:
            return None
        capacity = int(cfg.token_capacity or 0)
        evicting = capacity > 0 and any(len(chunk) > capacity for _, _, chunk in items)
        if evicting and (self._fused_reductions() is None or cfg.token_score_direction != "query_to_chunk"):
            return None
        p_len = len(prefix_ids)
        batch = max(1, int(cfg.score_batch_size or 1))
        by_len: Dict[int, List[int]] = {}
        for n, (_, _, chunk) in enumerate(items):
            by_len.setdefault(len(chunk), []).append(n)
        # kept positions: one scoring forward per group of same-length chunks, then the usual per-chunk selection
        keeps: List[Optional[List[int]]] = [None] * len(items)
        for c_len, members in by_len.items():
            if capacity <= 0 or c_len <= capacity:
                for n in members:
                    keeps[n] = self._keep_positions_for_chunk(prefix_ids, items[n][2], evict_q)
                continue
            for off in range(0, len(members), batch):
                part = members[off:off + batch]
                scored = self._chunk_head_scores_packed(prefix_ids, [items[n][2] for n in part], evict_q)
                for n, sc in zip(part, scored):
                    keeps[n] = self._keep_positions_for_chunk(prefix_ids, items[n][2], evict_q, sc)
        # destinations in cache order
        out: List[Optional[tuple]] = [None] * len(items)
        dsts, at = [], dst
        for n in range(len(items)):
            dsts.append(at)
            at += len(keeps[n])
        cache.slots(dst, at - dst)                                                  # capacity check
        # prefill: one packed forward per group, every sequence against the prefix KV, kept rows written to their slots
        for c_len, members in by_len.items():
            for off in range(0, len(members), batch):
                part = members[off:off + batch]
                rows_ids, rows_pos, slots = [], [], []
                for n in part:
                    order, ci, chunk = items[n]
                    c_start = self._chunk_rope_start(p_len, order, ci)
                    c_pos = self._range_positions(c_start, len(chunk))
                    ids, pos = chunk, c_pos
                    if cfg.cache_build_mode == "chunk_query":
                        tq_start = self._chunk_query_rope_start(p_len, c_start, len(chunk))
                        ids = chunk + window_q
                        pos = c_pos + self._range_positions(tq_start, len(window_q))
                    keep_set = set(keeps[n])
                    next_slot = iter(cache.slots(dsts[n], len(keeps[n])))
                    slots += [next(next_slot) if i in keep_set else -1 for i in range(len(chunk))] + [-1] * (len(ids) - len(chunk))
                    rows_ids.append(ids)
                    rows_pos.append(pos)
                    out[n] = (len(keeps[n]), [c_pos[i] for i in keeps[n]], keeps[n], c_start)
                if cfg.cache_build_mode == "chunk_query":
                    mask_args = self._mask_args(cfg.token_attention_mask, rows_before_chunk=0, chunk_len=c_len, query_len=len(window_q))
                else:
                    mask_args = dict(causal=False)
                self._forward_packed(rows_ids, rows_pos, cache=cache if p_len else None, ctx_len=p_len, store_slots=slots, want_logits=False,
                                     **mask_args)
        return out

    @torch.inference_mode()
    def build_prefill_cache(self, *, prefix_ids, context_ids, query_ids, scoring_query_ids=None):
        """Independent per-chunk prefill (cache_build_mode chunk_query / chunk_only) → (PagedCache, cache_positions, meta).

        Reference :2201-2328. Each selected chunk is forwarded against the prefix KV only (with the query window behind it
        in chunk_query mode) and only its kept rows are written to pages — eviction is the slot mapping, no gather."""
        cfg = self.config
        prefix_ids, context_ids, query_ids = list(prefix_ids), list(context_ids), list(query_ids)
        scoring_query_ids = list(scoring_query_ids if scoring_query_ids is not None else query_ids)
        if cfg.cache_build_mode in {"full_prompt_mask", "full_prompt_query"}:
            raise ValueError(f"{cfg.cache_build_mode} uses generate_full_prompt_mask instead of build_prefill_cache")
        if cfg.cache_build_mode not in {"chunk_query", "chunk_only"}:
            raise ValueError(f"Unsupported cache_build_mode: {cfg.cache_build_mode}")
        chunks, selected, scores, selection_q, mask = self._prepare_candidate_chunks(prefix_ids=prefix_ids, context_ids=context_ids,
                                                                                    scoring_query_ids=scoring_query_ids)
        evict_q = self._token_eviction_query_ids(scoring_query_ids, selection_q, mask)
        p_len = len(prefix_ids)
        capacity = p_len + sum(len(chunks[i]) for i in selected) + len(query_ids) + self.max_new_tokens + 2 * self.model.page_size
        cache = PagedCache(self, capacity)
        try:
            prefix_pos = self._range_positions(0, p_len)
            cache_positions: List[int] = []
            if prefix_ids:
                self._forward_packed([prefix_ids], [prefix_pos], causal=False, store_slots=cache.slots(0, p_len), want_logits=False)
                cache.length = p_len
                cache_positions.extend(prefix_pos)
            meta: List[FastDLLMChunkMeta] = []
            total_removed = 0
            window_q = self._window_query(selection_q, cfg.token_score_query_window)
            packed = self._prefill_chunks_packed(cache, cache.length, prefix_ids, [(order, ci, list(chunks[ci])) for order, ci in enumerate(selected)],
                                                 evict_q, window_q)
            for order, ci in enumerate(selected):
                chunk = list(chunks[ci])
                dst = cache.length
                if packed is not None:
                    kept, kept_pos, keep_union, c_start = packed[order]
                else:
                    kept, kept_pos, keep_union, c_start = self._prefill_one_chunk(cache, dst, prefix_ids, chunk, order, ci, evict_q, window_q)
                removed = max(0, len(chunk) - kept)
                total_removed += removed
                cache.length = dst + kept
                cache_positions.extend(kept_pos)
                meta.append(FastDLLMChunkMeta(chunk_index=ci, original_tokens=len(chunk), kept_tokens=kept, removed_tokens=removed,
                                              cache_start=dst, cache_end=dst + kept, rope_start=c_start, rope_end=c_start + len(chunk),
                                              score=scores.get(ci), kept_positions=list(keep_union)))
            cache.positions = list(cache_positions)
            q_start = self._final_query_rope_start(p_len, cache_positions, selected_count=len(selected))
        except BaseException:
            cache.release()
            raise
        return cache, cache_positions, {
            "selected_indices": selected, "chunk_scores": scores, "cache_build_mode": cfg.cache_build_mode, "prefix_tokens": p_len,
            "query_rope_start": q_start, "raw_context_tokens": len(context_ids), "candidate_chunks": len(chunks),
            "cache_tokens": cache.length, "removed_tokens": total_removed, "chunk_meta": meta,
        }

    @torch.inference_mode()
    def generate_from_cache(self, *, past_key_values: Optional[PagedCache], cache_positions: Sequence[int], query_ids, query_rope_start: int,
                            max_new_tokens: Optional[int] = None, diffusion_steps=None, force_diffusion: bool = False) -> List[int]:
        """Prefill the query on top of `past_key_values` (a PagedCache) and denoise block by block (reference :2678-2774)."""
        max_new = int(max_new_tokens if max_new_tokens is not None else self.max_new_tokens)
        if max_new <= 0:
            return []
        fixed_steps = None
        if force_diffusion or self.config.alg != "confidence_threshold":
            total_steps = int(diffusion_steps if diffusion_steps is not None else self.diffusion_steps)
            num_blocks = max(1, math.ceil(max_new / self.block_length))
            fixed_steps = max(1, math.ceil(total_steps / num_blocks))
        query_ids = list(query_ids)
        own = past_key_values is None
        cache = past_key_values if not own else PagedCache(self, len(query_ids) + max_new + self.model.page_size)
        try:
            if cache.length + len(query_ids) + max_new > cache.capacity:
                raise RuntimeError("paged cache too small for the query and the generation blocks")
            if not query_ids:
                raise ValueError("generate_from_cache needs a non-empty query")
            q_pos = self._range_positions(query_rope_start, len(query_ids))
            base = cache.length
            logits, _ = self._forward_packed([query_ids], [q_pos], causal=False, cache=cache if base else None, ctx_len=base,
                                             store_slots=cache.slots(base, len(query_ids)), logit_rows=[len(query_ids) - 1])
            cache.length = base + len(query_ids)
            return self._denoise_blocks(cache, suffix_pos_start=query_rope_start + len(query_ids), last_logit=logits[0],
                                        first_token=None, tail_in_cache=0, max_new=max_new, fixed_steps_per_block=fixed_steps,
                                        confidence_alg="origin" if force_diffusion else None)
        finally:
            if own:
                cache.release()

    # ------------------------------------------------------------------------------------------------ joint prefill
    def _prepare_candidate_chunks(self, *, prefix_ids, context_ids, scoring_query_ids):
        chunks = split_token_chunks(context_ids, self.config.chunk_size, split_from_tail=self.config.split_from_tail)
        chunks = [self._maybe_prepend_bos_to_chunk(c) for c in chunks]
        selected, scores, selection_q, mask = self.select_chunks(prefix_ids, chunks, scoring_query_ids)
        return chunks, selected, scores, selection_q, mask

    @torch.inference_mode()
    def generate_full_prompt_mask(self, *, prefix_ids, context_ids, query_ids, scoring_query_ids=None) -> FastDLLMParallelCompResult:
        """Select, evict, then ONE bidirectional prefill over [prefix ‖ kept chunk tokens ‖ query (‖ MASKs)] and block
        denoising (reference :2776-3024)."""
        t0 = time.time()
        cfg = self.config
        prefix_ids, context_ids, query_ids = list(prefix_ids), list(context_ids), list(query_ids)
        scoring_query_ids = list(scoring_query_ids if scoring_query_ids is not None else query_ids)
        chunks, selected, scores, selection_q, mask = self._prepare_candidate_chunks(prefix_ids=prefix_ids, context_ids=context_ids,
                                                                                    scoring_query_ids=scoring_query_ids)
        evict_q = self._token_eviction_query_ids(scoring_query_ids, selection_q, mask)
        p_len = len(prefix_ids)
        prompt_ids, prompt_pos = list(prefix_ids), self._range_positions(0, p_len)
        cache_positions = list(prompt_pos)
        meta: List[FastDLLMChunkMeta] = []
        total_removed, compressed_len = 0, p_len
        per_head = cfg.token_eviction_granularity == "per_head"
        spans: List[Tuple[int, int, List[torch.Tensor]]] = []
        for order, ci in enumerate(selected):
            chunk = list(chunks[ci])
            c_start = self._chunk_rope_start(p_len, order, ci)
            c_pos = self._range_positions(c_start, len(chunk))
            span_start = len(prompt_ids)
            if per_head:
                keep_ph = self._keep_positions_per_layer_per_head_for_chunk(prefix_ids, chunk, evict_q)
                keep = sorted({int(v) for k in keep_ph for v in k.reshape(-1).tolist()}) if keep_ph else []
                kept = int(keep_ph[0].shape[1]) if keep_ph else len(chunk)
                ids_in, pos_in, comp_pos = chunk, c_pos, c_pos[:kept]
            else:
                keep_ph = None
                keep = self._keep_positions_for_chunk(prefix_ids, chunk, evict_q)
                ids_in, pos_in = [chunk[i] for i in keep], [c_pos[i] for i in keep]
                kept, comp_pos = len(ids_in), pos_in
            prompt_ids.extend(ids_in)
            prompt_pos.extend(pos_in)
            if keep_ph is not None:
                spans.append((span_start, len(prompt_ids), keep_ph))
            removed = max(0, len(chunk) - kept)
            total_removed += removed
            meta.append(FastDLLMChunkMeta(chunk_index=ci, original_tokens=len(chunk), kept_tokens=kept, removed_tokens=removed,
                                          cache_start=compressed_len, cache_end=compressed_len + kept, rope_start=c_start,
                                          rope_end=c_start + len(chunk), score=scores.get(ci), kept_positions=list(keep)))
            cache_positions.extend(comp_pos)
            compressed_len += kept

        q_start = self._final_query_rope_start(p_len, cache_positions, selected_count=len(selected))
        full_q_start = self._final_query_rope_start(p_len, prompt_pos, selected_count=len(selected))
        max_new = int(self.max_new_tokens)
        mask_id = self._mask_token_id()
        full_prompt_len = len(prompt_ids) + len(query_ids)
        with_masks = cfg.cache_build_mode == "full_prompt_mask"
        blen0 = min(self.block_length, max_new)
        later0 = max_new - blen0
        full_ids = prompt_ids + query_ids + ([mask_id] * max_new if with_masks else [])
        full_pos = prompt_pos + self._range_positions(full_q_start, len(query_ids)) + (
            self._range_positions(full_q_start + len(query_ids), max_new) if with_masks else [])
        compacting = per_head and any(int(s[2][0].shape[1]) < (s[1] - s[0]) for s in spans)

        cache = PagedCache(self, len(full_ids) + self.model.page_size)
        try:
            # rows stored: prompt + query, then (full_prompt_mask) the later blocks' MASK slots; the first block's MASK rows
            # are the new rows of every denoise forward and are never stored
            if with_masks:
                slots = cache.slots(0, full_prompt_len) + [-1] * blen0 + cache.slots(full_prompt_len, later0)
            else:
                slots = cache.slots(0, full_prompt_len)
            logits, _ = self._forward_packed([full_ids], [full_pos], causal=False, store_slots=slots, logit_rows=[full_prompt_len - 1],
                                             store_unrotated_k=compacting)
            last_logit = logits[0]
            cache.length = full_prompt_len + (later0 if with_masks else 0)
            if compacting:
                # per-head eviction after the joint prefill (reference :2906-2912): keep lists cover prefix, kept chunk rows,
                # query and the stored MASK slots; compaction is in place, per layer and KV head
                seq_len = cache.length
                keep_global = self._full_prompt_keep_indices(seq_len=seq_len, spans=spans)
                for layer in range(self.arch.num_hidden_layers):
                    for kv in self.model.layer_cache(layer):
                        ops.compact_pages_per_head(kv, cache.page_ids, cache.page_ids, keep_global[layer], src_tokens=seq_len)
                cache.length = int(keep_global[0].shape[1])
                suffix_start = q_start + len(query_ids)
                # keys were stored un-rotated; they take the COMPACTED positions (reference :2890, :2912)
                stored_pos = list(cache_positions) + self._range_positions(q_start, len(query_ids))
                if with_masks:
                    stored_pos += self._range_positions(suffix_start + blen0, later0)
                assert len(stored_pos) == cache.length
                self.model.rope_rows(cache.page_ids, 0, stored_pos)
            else:
                suffix_start = full_q_start + len(query_ids)
            # un-shifted architectures take the first token from the first MASK slot's own row: the block loop's suffix
            # initialisation recomputes that row (and the MASK-slot K/V, with the same values) from the prompt K/V
            first = self._first_block_token(last_logit) if (with_masks and self.arch.logit_shift) else None
            fixed_steps = None
            if cfg.alg != "confidence_threshold":     # reference :2927-2929, :2977-2985
                fixed_steps = max(1, math.ceil(int(self.diffusion_steps) / max(1, math.ceil(max_new / self.block_length))))
            generated = self._denoise_blocks(cache, suffix_pos_start=suffix_start, last_logit=last_logit, first_token=first,
                                             tail_in_cache=later0 if with_masks else 0, max_new=max_new,
                                             fixed_steps_per_block=fixed_steps)
        finally:
            cache.release()

        self.total_generation_time += time.time() - t0
        eos = getattr(self.tokenizer, "eos_token_id", None)
        self.generated_token_num += sum(1 for t in generated if t != eos)
        return self._result(generated, selected, scores, cfg.cache_build_mode, p_len, len(query_ids), len(context_ids), len(chunks),
                            len(cache_positions), total_removed, meta)

    def _full_prompt_keep_indices(self, *, seq_len: int, spans) -> List[torch.Tensor]:
        """Per layer [Hkv, active_len] indices into the stored joint sequence (reference :2094-2127)."""
        out = []
        hkv = self.arch.num_key_value_heads
        for layer in range(self.arch.num_hidden_layers):
            heads = []
            for h in range(hkv):
                pieces, cursor = [], 0
                for start, end, keep_ph in spans:
                    if start > cursor:
                        pieces.append(torch.arange(cursor, start, device=self.device))
                    lk = keep_ph[min(layer, len(keep_ph) - 1)]
                    pieces.append(lk[min(h, lk.shape[0] - 1)].to(self.device) + start)
                    cursor = end
                if cursor < seq_len:
                    pieces.append(torch.arange(cursor, seq_len, device=self.device))
                heads.append(torch.cat(pieces))
            out.append(torch.stack(heads))
        return out

    # ------------------------------------------------------------------------------------------------ public entry points
    def _result(self, generated, selected, scores, mode, p_len, q_len, raw_ctx, n_chunks, cache_tokens, removed, meta):
        text = self.tokenizer.decode(generated, skip_special_tokens=False)
        eos = getattr(self.tokenizer, "eos_token", None)
        if eos and eos in text:
            text = text.split(eos)[0]
        return FastDLLMParallelCompResult(
            text=text, sequences=list(generated), selected_chunk_indices=list(selected), chunk_scores=dict(scores), cache_build_mode=mode,
            prefix_tokens=p_len, query_tokens=q_len, raw_context_tokens=raw_ctx, candidate_chunks=n_chunks, cache_tokens=cache_tokens,
            removed_tokens=removed, chunk_meta=meta, generation_blocks=max(1, math.ceil(self.max_new_tokens / self.block_length)),
            generation_block_length=self.block_length)

    @torch.inference_mode()
    def generate(self, *, prefix_ids, context_ids, query_ids, scoring_query_ids=None) -> FastDLLMParallelCompResult:
        mode = self.config.cache_build_mode
        if mode in {"full_prompt_mask", "full_prompt_query"}:
            return self.generate_full_prompt_mask(prefix_ids=prefix_ids, context_ids=context_ids, query_ids=query_ids,
                                                  scoring_query_ids=scoring_query_ids)
        if mode not in {"chunk_query", "chunk_only"}:
            raise ValueError(f"Unsupported cache_build_mode: {mode}")
        t0 = time.time()
        cache, cache_positions, meta = self.build_prefill_cache(prefix_ids=prefix_ids, context_ids=context_ids, query_ids=query_ids,
                                                                scoring_query_ids=scoring_query_ids)
        try:
            generated = self.generate_from_cache(past_key_values=cache, cache_positions=cache_positions, query_ids=query_ids,
                                                 query_rope_start=meta["query_rope_start"])
        finally:
            cache.release()
        self.total_generation_time += time.time() - t0
        eos = getattr(self.tokenizer, "eos_token_id", None)
        self.generated_token_num += sum(1 for t in generated if t != eos)
        return self._result(generated, meta["selected_indices"], meta["chunk_scores"], meta["cache_build_mode"], meta["prefix_tokens"],
                            len(list(query_ids)), meta["raw_context_tokens"], meta["candidate_chunks"], meta["cache_tokens"],
                            meta["removed_tokens"], meta["chunk_meta"])

    def encode_fragment(self, text: str) -> List[int]:
        return self.tokenizer.encode(text, add_special_tokens=False) if text else []

    def bos_ids(self) -> List[int]:
        return self._get_bos_token_ids() if self.config.add_bos_token else []

    def generate_from_text_parts(self, *, prefix: str, context: str, query: str, scoring_query: Optional[str] = None):
        return self.generate(prefix_ids=self.bos_ids() + self.encode_fragment(prefix), context_ids=self.encode_fragment(context),
                             query_ids=self.encode_fragment(query),
                             scoring_query_ids=self.encode_fragment(scoring_query if scoring_query is not None else query))


def _resolve_dtype(dtype):
    """prefilling_dllm_eval/fastdllm_v1_model.py:43-48."""
    if dtype in (None, "auto"):
        return dtype
    if isinstance(dtype, torch.dtype):
        return dtype
    return getattr(torch, str(dtype), torch.bfloat16)


def _load_tokenizer(path: str, trust_remote_code: bool):
    if not os.path.exists(os.path.join(path, "tokenizer.json")) and not os.path.exists(os.path.join(path, "tokenizer_config.json")):
        return None
    import transformers

    return transformers.AutoTokenizer.from_pretrained(path, trust_remote_code=trust_remote_code)


def load_fastdllm_parallelcomp(pretrained: str, fastdllm_dream_dir: Optional[str] = None, model_backend: str = "dream",
                               fastdllm_llada_dir: Optional[str] = None, **kwargs) -> FastDLLMParallelComp:
    """Same factory as the reference (:3113-3127). `fastdllm_dream_dir` is accepted and ignored: the model arithmetic is
    built in, there is no external model plug-in to import."""
    config = FastDLLMParallelCompConfig(fastdllm_dream_dir=fastdllm_dream_dir or "", model_backend=model_backend,
                                        fastdllm_llada_dir=fastdllm_llada_dir, pretrained=pretrained, **kwargs)
    return FastDLLMParallelComp(config)
