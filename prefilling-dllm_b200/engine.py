"""Prefill/decode (PD) engine facade over the paged model: the reference engine's boundary, field for field.

Mirrors `FastDLLMDreamEngine` (prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py:170-2556): the six PD methods
(`prefill_to_pd_record`, `snapshot_pd_record_kv`, `make_pd_record_from_kv_snapshot`, `make_pd_record_from_remote_engine`,
`decode_from_pd_record`, `release_pd_record`), the records they exchange (`DreamPrefillRecord :32-49`, `DreamKVSnapshot
:52-61`), the engine twins of chunk selection and per-head eviction (`select_chunks_by_engine :1154`,
`compute_prompt_keep_indices_per_layer_per_head :1325`, `generate_token_ids_from_chunk_local_kv :1683`) and the page
allocator with its whole-prompt prefix cache (`_PrefixPageAllocator :88-167`, here `model.PageAllocator`).

What differs in mechanism, not in result:
  * attention reads the prompt pages in place through the block table (no per-layer gather of the prompt KV, no mask
    tensor of [block, prompt + block]);
  * the LM head runs only on the rows whose logits are read (one row after a prefill, the label rows of a scoring
    forward) instead of on every row;
  * the unmask step is one kernel with one host read per step (reference :2135-2157 reads once per slot);
  * KV snapshots, loads and per-head compaction are page-copy kernels over all layers (reference: 2 x layers
    advanced-index gathers / scatters, staged through the CPU by default).
Sampling (temperature / top-k / top-p, reference :1658-1681) runs as eager steps on torch ops: the fused unmask kernel and the
captured step graph serve the greedy rule.
Not built (the arguments are accepted and rejected with NotImplementedError): the selection-dense variants of the sparse
prefill, tensor parallelism, the "distinct" KV layout for this facade.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from . import ops
from .model import denoise_blocks_batched, CachedPrefix, DreamArch, PageAllocator, PagedDreamModel, denoise_blocks, slots_for

_OFF = {"none", "off", "0", ""}
_DELTA_MODES = {"s4_left3", "delta_s4_left3", "sampled_delta_s4_left3"}


def _on_device(method):
    """Run an engine method with the engine's GPU as the current CUDA device (kernels launch on the current device)."""
    import functools

    @functools.wraps(method)
    def wrapper(self, *args, **kwargs):
        with torch.cuda.device(self.device):
            return method(self, *args, **kwargs)

    return wrapper


@dataclass
class FastDLLMEngineOutput:
    text: str
    token_ids: List[int]
    n_diff_steps: int


@dataclass
class DreamPrefillRecord:
    """Boundary state between prefill and decode (reference :32-49, same fields in the same order)."""

    prompt_ids: List[int]
    prompt_positions: List[int]
    suffix_positions: List[int]
    prompt_len: int
    full_prompt_len: int
    decode_len: int
    prompt_page_ids: List[int]
    block_page_ids: List[int]
    first_token_id: int
    last_context_logit: Optional[torch.Tensor]
    decode_delta_state: Optional[dict]
    owns_prompt_pages: bool
    cached_prefix: Optional[CachedPrefix] = None
    kv_mode: str = "full_dense"


@dataclass
class DreamKVSnapshot:
    """Transferable prompt KV payload (reference :52-61): per layer K and V as [prompt_len, Hkv, D]."""

    prompt_len: int
    page_size: int
    kv_mode: str
    k_by_layer: List[torch.Tensor]
    v_by_layer: List[torch.Tensor]
    last_context_logit: Optional[torch.Tensor] = None


@dataclass
class _EngineConfig:
    """The fields of the reference Config that callers of the facade read (config.py)."""

    model: str
    max_model_len: int
    max_num_batched_tokens: int
    max_num_seqs: int
    tensor_parallel_size: int
    device_start: int
    gpu_memory_utilization: float
    enforce_eager: bool
    kv_cache_layout: str
    mask_token_id: int
    diffusion_block_size: int
    num_kvcache_blocks: int
    kvcache_block_size: int
    model_name: str = "dream"
    model_type: str = "diffusion_lm"


class _TokenRun:
    """A run of tokens laid over a page list: what the block loop needs to know about a cache."""

    def __init__(self, page_ids: Sequence[int], length: int, page_size: int):
        self.page_ids, self.length, self.page_size = list(page_ids), int(length), int(page_size)

    def slots(self, start: int, n: int) -> List[int]:
        if start + n > len(self.page_ids) * self.page_size:
            raise RuntimeError("token run overflows its pages")
        return slots_for(self.page_ids, start, n, self.page_size)


class FastDLLMDreamEngine:
    """One model replica with its KV pool on one GPU; prefill and decode halves joined by a DreamPrefillRecord."""

    def __init__(self, model, *, max_model_len: int = 8192, block_length: int = 32, tensor_parallel_size: int = 1,
                 device_start: int = 0, gpu_memory_utilization: float = 0.60, max_num_batched_tokens: Optional[int] = None,
                 max_num_seqs: int = 1, mask_token_id: int = 151666, threshold: float = 0.9, temperature: float = 0.0,
                 top_p: Optional[float] = None, top_k: Optional[int] = None, enforce_eager: bool = True,
                 kv_cache_layout: str = "unified", master_port: int = 2333, shm_name: str = "prefilling_dllm_fastdllm",
                 dtype: Optional[torch.dtype] = None, num_kv_pages: Optional[int] = None, page_size: int = 256) -> None:
        """`model`: checkpoint directory (config.json + safetensors [+ tokenizer]) or a ready PagedDreamModel.
        Beyond the reference signature: `dtype` (default bf16), `num_kv_pages` (default: what fits in
        gpu_memory_utilization of the device after the weights) and `page_size` (reference Config default 256)."""
        self.block_length = int(block_length)
        self.mask_token_id = int(mask_token_id)
        self.threshold = float(threshold)
        self.temperature = float(temperature)
        self.top_p = top_p
        self.top_k = top_k
        if kv_cache_layout not in ("unified", "distinct"):
            raise ValueError(f"FastDLLMDreamEngine supports kv_cache_layout='unified' or 'distinct', got '{kv_cache_layout}'.")
        if kv_cache_layout != "unified":
            raise NotImplementedError("this facade keeps its pool in the unified layout; the distinct layout is served by the ops only")
        if int(tensor_parallel_size) != 1:
            raise NotImplementedError("tensor parallelism is not built: one replica per GPU, data parallel over requests")
        if not torch.cuda.is_available():
            raise RuntimeError("FastDLLMDreamEngine needs a CUDA device; there is no CPU path")
        self.tokenizer = None
        if isinstance(model, PagedDreamModel):
            self.model = model
            model_name = "<PagedDreamModel>"
        else:
            device = torch.device("cuda", int(device_start))
            dtype = dtype or torch.bfloat16
            arch = DreamArch.from_pretrained(model)
            if num_kv_pages is None:
                num_kv_pages = self._pages_that_fit(arch, device, dtype, page_size, gpu_memory_utilization)
            self.model = PagedDreamModel.from_pretrained(model, device=device, dtype=dtype, num_pages=int(num_kv_pages),
                                                         page_size=int(page_size), arch=arch)
            model_name = str(model)
            try:
                from transformers import AutoTokenizer

                self.tokenizer = AutoTokenizer.from_pretrained(model, use_fast=True, trust_remote_code=False)
            except Exception:  # ids in, ids out still works without a tokenizer; `text` is then empty
                self.tokenizer = None
        self.device = self.model.device
        self.page_size = self.model.page_size
        self._prefix_cache: PageAllocator = self.model.allocator
        self._active_decode_delta_state = None
        self.config = _EngineConfig(
            model=model_name, max_model_len=int(max_model_len), max_num_batched_tokens=int(max_num_batched_tokens or max_model_len),
            max_num_seqs=int(max_num_seqs), tensor_parallel_size=1, device_start=int(device_start),
            gpu_memory_utilization=float(gpu_memory_utilization), enforce_eager=bool(enforce_eager), kv_cache_layout="unified",
            mask_token_id=self.mask_token_id, diffusion_block_size=self.block_length, num_kvcache_blocks=self.model.num_pages,
            kvcache_block_size=self.page_size)

    @staticmethod
    def _pages_that_fit(arch: DreamArch, device, dtype, page_size: int, utilization: float) -> int:
        elem = torch.empty((), dtype=dtype).element_size()
        page_bytes = 2 * arch.num_hidden_layers * page_size * arch.num_key_value_heads * arch.head_dim * elem
        layer = (2 * arch.hidden_size * arch.hidden_size + 2 * arch.hidden_size * arch.num_key_value_heads * arch.head_dim
                 + 3 * arch.hidden_size * arch.intermediate_size)
        weight_bytes = (arch.num_hidden_layers * layer + 2 * arch.vocab_size * arch.hidden_size) * elem
        total = torch.cuda.get_device_properties(device).total_memory
        budget = int(total * float(utilization)) - weight_bytes - torch.cuda.memory_allocated(device)
        return max(4, budget // page_bytes)

    def close(self) -> None:
        self.model = None

    # ------------------------------------------------------------------------------------------------ forwards
    def _forward(self, ids, positions: Sequence[int], *, ctx_page_ids: Optional[Sequence[int]] = None, ctx_len: int = 0,
                 store_slots: Optional[Sequence[int]] = None, causal: bool = False, mask: Optional[torch.Tensor] = None,
                 logit_rows: Optional[Sequence[int]] = None, want_logits: bool = True, capture_layers=None, on_layer_stored=None,
                 attention_fn=None):
        """One sequence of new rows at `positions`, seeing the first `ctx_len` tokens held by `ctx_page_ids`."""
        m = self.model
        ids_t = ids if isinstance(ids, torch.Tensor) else m.ids_tensor(ids)
        n = int(ids_t.numel())
        if n != len(positions):
            raise ValueError(f"ids/positions length mismatch: {n} vs {len(positions)}")
        kwargs = {}
        if ctx_page_ids is not None and ctx_len > 0:
            kwargs = dict(block_table=m.i32(list(ctx_page_ids)).view(1, -1), seq_lens=m.i32([ctx_len + n]), max_seq_len=ctx_len + n)
        with torch.cuda.device(self.device):
            return m.forward(ids_t, torch.tensor(list(positions), dtype=torch.long, device=m.device), cu_seqlens=m.i32([0, n]),
                             max_query_len=n, slot_mapping=None if store_slots is None else m.i32(list(store_slots)),
                             causal=causal, new_row_mask=mask, logit_rows=None if logit_rows is None else m.ids_tensor(logit_rows),
                             want_logits=want_logits, capture_qk_layers=capture_layers, on_layer_stored=on_layer_stored,
                             attention_fn=attention_fn, **kwargs)

    def _selection_mask(self, mode: str, *, seq_len: int, prefix_len: int, chunk_len: int, query_len: int):
        """(causal flag, dense mask or None) for a selection forward (reference _selection_prefill_mask :930-953)."""
        mode = (mode or "full").lower()
        if mode in {"full", "none"}:
            return False, None
        if mode == "causal":
            return True, None
        if mode == "query_to_chunk":
            mask = torch.ones((seq_len, seq_len), dtype=torch.bool, device=self.device)
            q_start = prefix_len + chunk_len
            if query_len > 0 and q_start < seq_len:
                mask[prefix_len:q_start, q_start:] = False
            return False, mask
        raise ValueError(f"Unsupported selection attention mask: {mode}")

    # ------------------------------------------------------------------------------------------------ KV movement
    def _layer_pools(self):
        """The pool seen as one unified cache of 2 * layers * pages pages, so one page list addresses every layer."""
        kv = self.model.kv_cache                     # [2, layers, pages, page_size, Hkv, D]
        return kv.view(2 * kv.shape[1] * kv.shape[2], kv.shape[3], kv.shape[4], kv.shape[5])

    def _all_layer_page_ids(self, page_ids: Sequence[int]) -> torch.Tensor:
        """Page ids of `page_ids` in every (k|v, layer) plane of `_layer_pools()`, plane-major."""
        kv = self.model.kv_cache
        planes, pages = 2 * kv.shape[1], kv.shape[2]
        base = torch.tensor(list(page_ids), dtype=torch.int32, device=self.device)
        offsets = torch.arange(planes, dtype=torch.int32, device=self.device) * pages
        return (offsets.view(-1, 1) + base.view(1, -1)).reshape(-1).contiguous()

    def _normalize_per_head_keep_indices(self, keep_indices_per_layer_per_head, *, full_prompt_len: int) -> Tuple[List[torch.Tensor], int]:
        """Validation of reference :560-605, same messages."""
        kv = self.model.kv_cache
        num_layers, num_heads = int(kv.shape[1]), int(kv.shape[4])
        if len(keep_indices_per_layer_per_head) != num_layers:
            raise ValueError("per-head keep index layer count mismatch: "
                             f"got {len(keep_indices_per_layer_per_head)}, expected {num_layers}")
        normalized: List[torch.Tensor] = []
        active_len: Optional[int] = None
        for layer_idx, layer_keep in enumerate(keep_indices_per_layer_per_head):
            keep = torch.as_tensor(layer_keep, dtype=torch.long, device=self.device)
            if keep.ndim != 2:
                raise ValueError(f"Layer {layer_idx} keep indices must be [num_heads, active_len], got {tuple(keep.shape)}")
            if int(keep.shape[0]) != num_heads:
                raise ValueError(f"Layer {layer_idx} keep head count mismatch: got {keep.shape[0]}, expected {num_heads}")
            if active_len is None:
                active_len = int(keep.shape[1])
            elif int(keep.shape[1]) != active_len:
                raise ValueError(f"Layer {layer_idx} active length mismatch: got {keep.shape[1]}, expected {active_len}")
            if keep.numel() > 0 and (int(keep.min().item()) < 0 or int(keep.max().item()) >= full_prompt_len):
                raise ValueError(f"Layer {layer_idx} keep indices are outside full prompt length {full_prompt_len}.")
            normalized.append(keep.contiguous())
        return normalized, int(active_len or 0)

    def _compact_prompt_cache_per_layer_per_head(self, prompt_page_ids: List[int], keep_indices_per_layer_per_head, *,
                                                 src_tokens: Optional[int] = None) -> int:
        """In-place compaction of the kept tokens to the front of the prompt pages, per layer and KV head (:607-638)."""
        if not keep_indices_per_layer_per_head:
            return 0
        active_len = int(keep_indices_per_layer_per_head[0].shape[1])
        if active_len <= 0:
            return 0
        src_tokens = int(src_tokens if src_tokens is not None else len(prompt_page_ids) * self.page_size)
        for layer_idx, keep in enumerate(keep_indices_per_layer_per_head):
            for cache in self.model.layer_cache(layer_idx):
                ops.compact_pages_per_head(cache, prompt_page_ids, prompt_page_ids, keep, src_tokens=src_tokens)
        return active_len

    def _copy_chunk_local_kv_to_prompt_pages(self, *, src_page_ids: List[int], dst_page_ids: List[int], src_chunk_start: int,
                                             dst_start: int, keep_indices_per_layer_per_head) -> int:
        """Kept tokens of a locally prefilled chunk → `dst_start...` of the prompt pages, per layer and KV head (:525-558)."""
        if not keep_indices_per_layer_per_head:
            return 0
        keep_count = int(keep_indices_per_layer_per_head[0].shape[1])
        if keep_count <= 0:
            return 0
        src_tokens = len(src_page_ids) * self.page_size
        for layer_idx, keep in enumerate(keep_indices_per_layer_per_head):
            if int(keep.shape[1]) != keep_count:
                raise ValueError(f"Layer {layer_idx} keep_count mismatch in chunk-local KV copy")
            for cache in self.model.layer_cache(layer_idx):
                ops.compact_pages_per_head(cache, src_page_ids, dst_page_ids, keep + int(src_chunk_start), src_tokens=src_tokens,
                                           dst_start=int(dst_start))
        return keep_count

    def _gather_prompt_pages_all_layers(self, prompt_page_ids: Sequence[int], prompt_len: int) -> torch.Tensor:
        """[2, layers, n_pages * page_size, Hkv, D]: every layer's K and V of the prompt pages, ONE gather launch."""
        kv = self.model.kv_cache
        n_pages = math.ceil(prompt_len / self.page_size)
        ids = self._all_layer_page_ids(list(prompt_page_ids)[:n_pages])
        with torch.cuda.device(self.device):
            dense = ops.gather_pages(self._layer_pools(), ids, int(ids.numel()) * self.page_size)
        return dense.view(2, kv.shape[1], n_pages * self.page_size, kv.shape[4], kv.shape[5])

    def _snapshot_prompt_cache_per_layer(self, prompt_page_ids: List[int], prompt_len: int) -> Tuple[List[torch.Tensor], List[torch.Tensor]]:
        if prompt_len <= 0:
            return [], []
        dense = self._gather_prompt_pages_all_layers(prompt_page_ids, prompt_len)
        layers = dense.shape[1]
        return [dense[0, i, :prompt_len] for i in range(layers)], [dense[1, i, :prompt_len] for i in range(layers)]

    def _load_prompt_cache_per_layer(self, prompt_page_ids: List[int], prompt_len: int, k_by_layer, v_by_layer) -> None:
        """Per-layer [prompt_len, Hkv, D] tensors → the prompt pages of every layer, ONE scatter launch (:664-698)."""
        if prompt_len <= 0:
            return
        kv = self.model.kv_cache
        layers = int(kv.shape[1])
        if len(k_by_layer) != layers or len(v_by_layer) != layers:
            raise ValueError(f"PD KV snapshot layer count mismatch: k={len(k_by_layer)} v={len(v_by_layer)} expected={layers}")
        expected = (int(prompt_len), int(kv.shape[4]), int(kv.shape[5]))
        for layer_idx, (layer_k, layer_v) in enumerate(zip(k_by_layer, v_by_layer)):
            if tuple(layer_k.shape) != expected or tuple(layer_v.shape) != expected:
                raise ValueError(f"PD KV snapshot shape mismatch at layer {layer_idx}: "
                                 f"k={tuple(layer_k.shape)} v={tuple(layer_v.shape)} expected={expected}")
        n_pages = math.ceil(prompt_len / self.page_size)
        padded = n_pages * self.page_size
        with torch.cuda.device(self.device):
            staged = torch.zeros((2, layers, padded) + expected[1:], dtype=kv.dtype, device=self.device)
            for plane, tensors in enumerate((k_by_layer, v_by_layer)):
                for layer_idx, t in enumerate(tensors):
                    staged[plane, layer_idx, :prompt_len].copy_(t, non_blocking=True)
            ids = self._all_layer_page_ids(list(prompt_page_ids)[:n_pages])
            ops.scatter_pages(staged.view(-1, expected[1], expected[2]), self._layer_pools(), ids)

    @_on_device
    def snapshot_pd_record_kv(self, record: DreamPrefillRecord, *, device="cpu") -> DreamKVSnapshot:
        """Copy the prompt KV a record refers to into fresh tensors on `device` (reference :700-726)."""
        target = torch.device(device)
        if target.type == "cuda" and target.index is None:
            target = torch.device("cuda", torch.cuda.current_device())
        k_by_layer: List[torch.Tensor] = []
        v_by_layer: List[torch.Tensor] = []
        if record.prompt_len > 0:
            dense = self._gather_prompt_pages_all_layers(record.prompt_page_ids, record.prompt_len)
            if target != self.device:
                dense = dense.to(device=target)      # one copy for all layers
            layers = dense.shape[1]
            k_by_layer = [dense[0, i, :record.prompt_len] for i in range(layers)]
            v_by_layer = [dense[1, i, :record.prompt_len] for i in range(layers)]
        last = record.last_context_logit
        if last is not None:
            last = last.detach().to(device=target).contiguous()
        return DreamKVSnapshot(prompt_len=record.prompt_len, page_size=self.page_size, kv_mode=record.kv_mode, k_by_layer=k_by_layer,
                               v_by_layer=v_by_layer, last_context_logit=last)

    def _allocate_prompt_and_block_pages(self, prompt_len: int, decode_len: int) -> Tuple[List[int], List[int]]:
        n_prompt = math.ceil(prompt_len / self.page_size)
        n_block = math.ceil(decode_len / self.page_size)
        self._prefix_cache.ensure_free(n_prompt + n_block)
        prompt_pages = self._prefix_cache.allocate_pages(n_prompt)
        try:
            block_pages = self._prefix_cache.allocate_pages(n_block)
        except BaseException:
            self._prefix_cache.release_pages(prompt_pages)
            raise
        return prompt_pages, block_pages

    def _record_like(self, source: DreamPrefillRecord, prompt_page_ids, block_page_ids, last_context_logit, decode_delta_state):
        return DreamPrefillRecord(
            prompt_ids=list(source.prompt_ids), prompt_positions=list(source.prompt_positions),
            suffix_positions=list(source.suffix_positions), prompt_len=source.prompt_len, full_prompt_len=source.full_prompt_len,
            decode_len=source.decode_len, prompt_page_ids=prompt_page_ids, block_page_ids=block_page_ids,
            first_token_id=source.first_token_id, last_context_logit=last_context_logit, decode_delta_state=decode_delta_state,
            owns_prompt_pages=True, cached_prefix=None, kv_mode=source.kv_mode)

    @_on_device
    def make_pd_record_from_kv_snapshot(self, source: DreamPrefillRecord, snapshot: DreamKVSnapshot) -> DreamPrefillRecord:
        """Allocate local pages, load a snapshot into them, return a decode-ready record (reference :728-781)."""
        if snapshot.page_size != self.page_size:
            raise ValueError(f"PD KV snapshot page_size mismatch: snapshot={snapshot.page_size}, engine={self.page_size}")
        if snapshot.prompt_len != source.prompt_len:
            raise ValueError(f"PD KV snapshot prompt_len mismatch: snapshot={snapshot.prompt_len}, source={source.prompt_len}")
        if snapshot.kv_mode != source.kv_mode:
            raise ValueError(f"PD KV snapshot mode mismatch: snapshot={snapshot.kv_mode}, source={source.kv_mode}")
        prompt_pages, block_pages = self._allocate_prompt_and_block_pages(source.prompt_len, source.decode_len)
        try:
            self._load_prompt_cache_per_layer(prompt_pages, source.prompt_len, snapshot.k_by_layer, snapshot.v_by_layer)
        except BaseException:
            self._prefix_cache.release_pages(prompt_pages + block_pages)
            raise
        last = snapshot.last_context_logit
        if last is not None:
            last = last.to(device=self.device).contiguous()
        return self._record_like(source, prompt_pages, block_pages, last, source.decode_delta_state)

    @_on_device
    def make_pd_record_from_remote_engine(self, source_engine: "FastDLLMDreamEngine", source: DreamPrefillRecord, *,
                                          non_blocking: bool = True) -> DreamPrefillRecord:
        """Copy prompt KV from another engine's pool (same or another GPU) into this one (reference :800-881).

        ONE kernel on this GPU reads the source pages of every layer through peer access (across NVLink when the engines
        sit on different GPUs) and writes them into the freshly allocated local pages — no staging buffer, instead of
        2 x layers gathers, copies and scatters. `non_blocking` is accepted for signature parity: the copy is always
        asynchronous on this device's current stream, ordered after the source device's current stream."""
        if self.page_size != source_engine.page_size:
            raise ValueError(f"remote-engine PD page_size mismatch: source={source_engine.page_size}, target={self.page_size}")
        src_kv, dst_kv = source_engine.model.kv_cache, self.model.kv_cache
        if int(src_kv.shape[1]) != int(dst_kv.shape[1]):
            raise ValueError(f"remote-engine PD layer mismatch: source={int(src_kv.shape[1])}, target={int(dst_kv.shape[1])}")
        prompt_len = int(source.prompt_len)
        prompt_pages, block_pages = self._allocate_prompt_and_block_pages(prompt_len, source.decode_len)
        try:
            if prompt_len > 0:
                n_pages = math.ceil(prompt_len / self.page_size)
                planes = 2 * int(dst_kv.shape[1])
                src_ids = source_engine._all_layer_page_ids(source.prompt_page_ids[:n_pages]).to(self.device)
                dst_ids = self._all_layer_page_ids(prompt_pages[:n_pages])
                if src_kv.dtype != dst_kv.dtype:
                    raise ValueError(f"remote-engine PD dtype mismatch: source={src_kv.dtype}, target={dst_kv.dtype}")
                # the source must have finished writing these pages before this GPU reads them
                if source_engine.device != self.device:
                    done = torch.cuda.Event()
                    done.record(torch.cuda.current_stream(source_engine.device))
                    torch.cuda.current_stream(self.device).wait_event(done)
                ops.copy_pages(source_engine._layer_pools(), src_ids, self._layer_pools(), dst_ids, n_lists=planes, tokens_per_list=prompt_len)
                # ... and must not reuse them before this GPU has read them: the copy kernel runs on THIS device's stream, so
                # a release_pd_record(source) followed by a new prefill on the source would otherwise overwrite pages that are
                # still being read across NVLink. Later work on the source's current stream is ordered after the copy.
                if source_engine.device != self.device:
                    copied = torch.cuda.Event()
                    copied.record(torch.cuda.current_stream(self.device))
                    torch.cuda.current_stream(source_engine.device).wait_event(copied)
        except BaseException:
            self._prefix_cache.release_pages(prompt_pages + block_pages)
            raise
        last = source.last_context_logit
        if last is not None:
            last = last.to(device=self.device).contiguous()
        return self._record_like(source, prompt_pages, block_pages, last, self._delta_state_on(source.decode_delta_state, self.device))

    @staticmethod
    def _delta_state_on(state: Optional[dict], device) -> Optional[dict]:
        """A record's decode-delta state with its full-prompt KV on `device` (reference :784-798)."""
        if state is None:
            return None
        moved = dict(state)
        for key in ("full_k", "full_v"):
            if moved.get(key) is not None:
                moved[key] = [None if t is None else t.to(device=device).contiguous() for t in moved[key]]
        return moved

    # ------------------------------------------------------------------------------------------------ prefill half
    @staticmethod
    def _check_modes(*, prefill_sparse_mode, prefill_delta_mode, prefill_delta_selection_mode, prefill_delta_direction,
                              decode_delta_mode, has_keep: bool) -> None:
        """Argument checks of reference :1924-1935, :2012-2017, :2074-2075, and the refusal of the one mode that is not built."""
        sparse = (prefill_sparse_mode or "none").lower()
        use_sparse = sparse not in _OFF
        if use_sparse and sparse != "eviction_mask":
            raise ValueError(f"Unsupported prefill_sparse_mode: {sparse}")
        if use_sparse and not has_keep:
            raise ValueError("prefill_sparse_mode=eviction_mask requires prompt_keep_indices_per_layer_per_head.")
        if use_sparse:
            if (prefill_delta_mode or "none").lower() not in _OFF | {"s4_left3", "delta_s4_left3", "sampled_delta_s4_left3"}:
                raise ValueError(f"Unsupported prefill_delta_mode: {prefill_delta_mode}")
            if (prefill_delta_selection_mode or "none").lower() not in _OFF | {"selection_dense_replace", "selection_dense_add"}:
                raise ValueError(f"Unsupported prefill_delta_selection_mode: {prefill_delta_selection_mode}")
            if (prefill_delta_direction or "left").lower() not in {"left", "right", "both"}:
                raise ValueError(f"Unsupported prefill_delta_direction: {prefill_delta_direction}")
            if (prefill_delta_selection_mode or "none").lower() not in _OFF:
                raise NotImplementedError("prefill_delta_selection_mode (anchor outputs reused from the selection pass) is not built")
        delta = (decode_delta_mode or "none").lower()
        if delta not in _OFF | _DELTA_MODES and has_keep and not use_sparse:
            raise ValueError(f"Unsupported decode_delta_mode: {delta}")

    @_on_device
    @torch.inference_mode()
    def prefill_to_pd_record(self, prompt_ids: Sequence[int], *, max_new_tokens: int, prompt_positions: Optional[Sequence[int]] = None,
                             active_prompt_positions: Optional[Sequence[int]] = None,
                             prompt_keep_indices_per_layer_per_head=None, decode_delta_mode: str = "none", decode_delta_stride: int = 4,
                             decode_delta_left: int = 3, decode_delta_scale: float = 1.0, decode_delta_debug: bool = False,
                             prefill_sparse_mode: str = "none", prefill_delta_mode: str = "none", prefill_delta_stride: int = 8,
                             prefill_delta_left: int = 7, prefill_delta_right: int = 0, prefill_delta_direction: str = "left",
                             prefill_delta_scale: float = 1.0, prefill_delta_debug: bool = False,
                             prefill_delta_selection_mode: str = "none", prefill_delta_selection_scale: float = 1.0,
                             prefill_selection_dense_outputs: Optional[dict] = None, kv_stream=None) -> DreamPrefillRecord:
        """Prefill `[prompt ‖ MASK x block_length]` (or `MASK x max_new_tokens` for several blocks) bidirectionally into pages
        and return the decode-ready boundary state (reference :1879-2108). With keep indices the prompt KV is compacted per layer and KV head after the prefill
        ("compacted_posthoc_eviction"); without them the whole prompt is registered in the prefix cache and reused by
        the next request with the same prompt ids.
        `kv_stream` (not in the reference): a `pd_wire.KVStreamWriter`; the prompt KV is then sent layer group by layer group
        WHILE the prefill runs (full-dense records only)."""
        if max_new_tokens <= 0:
            raise ValueError("prefill_to_pd_record requires max_new_tokens > 0")
        if kv_stream is not None and prompt_keep_indices_per_layer_per_head is not None:
            raise ValueError("kv_stream carries full_dense records only: per-head eviction rewrites the pages after the prefill")
        prompt_ids = [int(x) for x in prompt_ids]
        prompt_positions = list(range(len(prompt_ids))) if prompt_positions is None else [int(x) for x in prompt_positions]
        if len(prompt_ids) != len(prompt_positions):
            raise ValueError(f"prompt_ids/prompt_positions length mismatch: {len(prompt_ids)} vs {len(prompt_positions)}")
        # One block: the reference's record, MASK slots padded to the block length. More than one block (the reference stops
        # here with NotImplementedError, fastdllm_engine.py:1911-1915): the record carries max_new_tokens MASK slots, all of
        # them in the joint prefill, as the eval class's full_prompt_mask flow does (fastdllm_parallelcomp.py:2896-2912).
        decode_len = self.block_length if max_new_tokens <= self.block_length else int(max_new_tokens)
        has_keep = prompt_keep_indices_per_layer_per_head is not None
        self._check_modes(prefill_sparse_mode=prefill_sparse_mode, prefill_delta_mode=prefill_delta_mode,
                                   prefill_delta_selection_mode=prefill_delta_selection_mode,
                                   prefill_delta_direction=prefill_delta_direction, decode_delta_mode=decode_delta_mode, has_keep=has_keep)
        keep: Optional[List[torch.Tensor]] = None
        active_len: Optional[int] = None
        if has_keep:
            keep, active_len = self._normalize_per_head_keep_indices(prompt_keep_indices_per_layer_per_head, full_prompt_len=len(prompt_ids))
            if active_prompt_positions is None:
                raise ValueError("active_prompt_positions is required for per-head KV eviction.")
            active_prompt_positions = [int(x) for x in active_prompt_positions]
            if len(active_prompt_positions) != active_len:
                raise ValueError("active_prompt_positions length mismatch: "
                                 f"{len(active_prompt_positions)} vs per-head active length {active_len}")
        elif active_prompt_positions is not None:
            raise ValueError("active_prompt_positions requires prompt_keep_indices_per_layer_per_head.")

        prefill_suffix_start = (max(prompt_positions) + 1) if prompt_positions else 0
        prefill_suffix_positions = list(range(prefill_suffix_start, prefill_suffix_start + decode_len))
        use_sparse = (prefill_sparse_mode or "none").lower() not in _OFF
        if keep is not None and not use_sparse:
            suffix_start = (max(active_prompt_positions) + 1) if active_prompt_positions else 0
            suffix_positions = list(range(suffix_start, suffix_start + decode_len))
            prompt_len, full_prompt_len, kv_mode = int(active_len or 0), len(prompt_ids), "compacted_posthoc_eviction"
        else:
            # dense prefill, or a prefill whose attention is restricted to the kept keys: the whole prompt KV stays in pages
            suffix_positions = prefill_suffix_positions
            prompt_len = full_prompt_len = len(prompt_ids)
            kv_mode = "full_prefill_sparse_delta" if use_sparse else "full_dense"
        if full_prompt_len + decode_len > self.config.max_model_len:
            raise ValueError(f"full_prompt_mask length {full_prompt_len + decode_len} exceeds max_model_len={self.config.max_model_len}")

        n_prompt_pages = math.ceil(full_prompt_len / self.page_size)
        n_block_pages = math.ceil(decode_len / self.page_size)
        use_prefix_cache = keep is None
        # the prompt KV of a joint prefill depends on how many MASK slots it saw: records of several blocks get entries of
        # their own in the prefix cache
        cache_key = prompt_ids if decode_len == self.block_length else prompt_ids + [-decode_len]
        cached = self._prefix_cache.lookup_prefix(cache_key) if use_prefix_cache else None
        owns_prompt_pages = False
        decode_delta_state: Optional[dict] = None
        stream_header = dict(prompt_ids=prompt_ids, prompt_positions=prompt_positions, suffix_positions=suffix_positions,
                             full_prompt_len=full_prompt_len, decode_len=decode_len, kv_mode=kv_mode) if kv_stream is not None else None
        if cached is not None:
            prompt_page_ids = cached.page_ids
            cached.ref_count += 1
            last_context_logit = cached.last_context_logit
            if kv_stream is not None:        # nothing is computed on a prefix-cache hit: the pages are final already
                kv_stream.begin(prompt_page_ids=prompt_page_ids, prompt_len=prompt_len, header=stream_header)
                for layer in range(self.model.arch.num_hidden_layers):
                    kv_stream.on_layer_stored(layer)
            try:
                self._prefix_cache.ensure_free(n_block_pages)
                block_page_ids = self._prefix_cache.allocate_pages(n_block_pages)
            except BaseException:
                cached.ref_count -= 1
                raise
            # the reference runs an all-MASK replace forward here (:2088-2094) and reads only row 0 of its SHIFTED logits,
            # which is the cached last-context logit: the forward changes nothing, so it is not run
            first_token = self._first_token(last_context_logit)
        else:
            self._prefix_cache.ensure_free(n_prompt_pages + n_block_pages)
            prompt_page_ids = self._prefix_cache.allocate_pages(n_prompt_pages)
            try:
                block_page_ids = self._prefix_cache.allocate_pages(n_block_pages)
            except BaseException:
                self._prefix_cache.release_pages(prompt_page_ids)
                raise
            owns_prompt_pages = not use_prefix_cache
            try:
                if full_prompt_len <= 0:
                    raise ValueError("prefill_to_pd_record needs at least one prompt token")
                full_ids = prompt_ids + [self.mask_token_id] * decode_len
                slots = slots_for(prompt_page_ids, 0, full_prompt_len, self.page_size) + slots_for(block_page_ids, 0, decode_len, self.page_size)
                # Dream reads token p from logits[p - 1]: the first block token and the "last context logit" are both the
                # row of the last prompt token, the only row the LM head is run on. An un-shifted architecture (LLaDA) reads
                # token p from logits[p]: the row kept is the first MASK slot's own, which is also what the all-MASK
                # replace forward of a prefix-cache hit would give for that slot. (The reference engine has no un-shifted
                # model; this follows its eval class, fastdllm_parallelcomp.py:1017-1024, 2385-2397.)
                first_row = full_prompt_len - 1 if self.model.arch.logit_shift else full_prompt_len
                if kv_stream is not None:
                    kv_stream.begin(prompt_page_ids=prompt_page_ids, prompt_len=prompt_len, header=stream_header)
                sparse_attention = None
                if use_sparse:
                    stride = max(1, int(prefill_delta_stride or 1))
                    direction = (prefill_delta_direction or "left").lower()
                    sparse_attention = self._sparse_prefill_attention(
                        keep, full_prompt_len=full_prompt_len, seq_len=full_prompt_len + decode_len,
                        delta=(prefill_delta_mode or "none").lower() in _DELTA_MODES, stride=stride, left=max(0, int(prefill_delta_left)),
                        right=max(0, int(prefill_delta_right)), direction=direction,
                        anchor_offset=0 if direction == "right" else stride - 1, scale=float(prefill_delta_scale))
                logits, _ = self._forward(full_ids, list(prompt_positions) + prefill_suffix_positions, store_slots=slots,
                                          logit_rows=[first_row], on_layer_stored=None if kv_stream is None else kv_stream.on_layer_stored,
                                          attention_fn=sparse_attention)
                last_context_logit = logits[0].detach()
                first_token = self._first_token(last_context_logit)
                if keep is not None and not use_sparse:
                    if (decode_delta_mode or "none").lower() in _DELTA_MODES:
                        if decode_len != self.block_length:
                            raise NotImplementedError("the decode delta correction serves one-block records")
                        # the un-evicted prompt KV, kept beside the record: decode corrects every stride-th block row with dense
                        # attention over it (reference :2059-2073)
                        full = self._snapshot_prompt_cache_per_layer(prompt_page_ids, full_prompt_len)
                        stride = max(1, int(decode_delta_stride or 4))
                        decode_delta_state = {"enabled": True, "mode": "s4_left3", "full_k": full[0], "full_v": full[1],
                                              "full_prompt_len": full_prompt_len, "active_prompt_len": int(active_len or 0), "stride": stride,
                                              "left": max(0, int(decode_delta_left)), "anchor_offset": stride - 1,
                                              "scale": float(decode_delta_scale), "debug": bool(decode_delta_debug)}
                    self._compact_prompt_cache_per_layer_per_head(prompt_page_ids, keep, src_tokens=full_prompt_len)
                    active_pages = math.ceil(prompt_len / self.page_size)
                    if active_pages < len(prompt_page_ids):
                        self._prefix_cache.release_pages(prompt_page_ids[active_pages:])
                        prompt_page_ids = prompt_page_ids[:active_pages]
                ops.check_status(self.device)
            except BaseException:
                self._prefix_cache.release_pages(block_page_ids)
                self._prefix_cache.release_pages(prompt_page_ids)
                raise
            if use_prefix_cache:
                self._prefix_cache.register_prefix(cache_key, prompt_page_ids, prompt_len, last_context_logit)
        record = DreamPrefillRecord(
            prompt_ids=prompt_ids, prompt_positions=prompt_positions, suffix_positions=suffix_positions, prompt_len=prompt_len,
            full_prompt_len=full_prompt_len, decode_len=decode_len, prompt_page_ids=prompt_page_ids, block_page_ids=block_page_ids,
            first_token_id=first_token, last_context_logit=last_context_logit, decode_delta_state=decode_delta_state,
            owns_prompt_pages=owns_prompt_pages, cached_prefix=cached, kv_mode=kv_mode)
        if kv_stream is not None:
            kv_stream.finish(record)
        return record

    # ------------------------------------------------------------------------------------------------ decode half
    def _denoise_block(self, *, ctx_page_ids: Sequence[int], ctx_len: int, block_slots: Sequence[int], block_positions: Sequence[int],
                       first_token_id: int, last_context_logit: Optional[torch.Tensor]) -> Tuple[torch.Tensor, int]:
        """Confidence-threshold denoising of one block against `ctx_len` cached tokens (reference :2133-2157): every
        step forwards the whole block (its K/V replace their slots), softmax in fp32, the most confident masked slot is
        always accepted and every other one whose confidence reaches the threshold."""
        decode_len = len(block_positions)
        n_steps = 0
        remaining = decode_len - 1
        if self._uses_sampler():
            # eager steps: the forward through the C-ABI kernels, the sampler and the transfer rule on torch ops
            block = torch.full((decode_len,), self.mask_token_id, dtype=torch.long, device=self.device)
            block[0] = int(first_token_id)
            while remaining > 0:
                n_steps += 1
                if n_steps > decode_len + 8:
                    raise RuntimeError("denoising did not converge: every step must unmask at least one slot")
                logits, _ = self._forward(block, block_positions, ctx_page_ids=ctx_page_ids, ctx_len=ctx_len, store_slots=block_slots)
                remaining = self._sampled_unmask(logits, block, last_context_logit)
            return block.clone(), n_steps
        runner = self.model.block_step_runner(block_len=decode_len, positions=block_positions, ctx_page_ids=ctx_page_ids, ctx_len=ctx_len,
                                              mask_token_id=self.mask_token_id, threshold=self.threshold, last_logit=last_context_logit,
                                              shift=self.model.arch.logit_shift, softmax_dtype=torch.float32, store_slots=block_slots,
                                              use_graph=not self.config.enforce_eager)
        block = runner.block                          # the step's ids buffer, updated in place by the unmask kernel
        block.fill_(self.mask_token_id)
        block[0] = int(first_token_id)
        while remaining > 0:
            n_steps += 1
            remaining = runner.run()      # forward + unmask kernel (CUDA graph replays unless enforce_eager); one host read
            if n_steps > decode_len + 8:
                raise RuntimeError("denoising did not converge: every step must unmask at least one slot")
        return block.clone(), n_steps

    @staticmethod
    def _spread_rows(anchors: Sequence[int], seq_len: int, *, left: int, right: int, direction: str):
        """(row, anchor index) pairs of the strided correction (reference attention_v4.py:145-158, :274-288): the delta measured
        at an anchor row is added to the rows of its window — [anchor - left, anchor] ("left"), [anchor, anchor + right]
        ("right") or both sides — clipped to the sequence."""
        rows, which = [], []
        for idx, a in enumerate(anchors):
            lo = a if direction == "right" else max(0, a - left)
            hi = a if direction == "left" else min(seq_len - 1, a + right)
            for r in range(lo, hi + 1):
                rows.append(r)
                which.append(idx)
        return rows, which

    def _apply_delta(self, out: torch.Tensor, dense: torch.Tensor, *, stride: int, left: int, right: int, direction: str,
                     anchor_offset: int, scale: float) -> None:
        """out += spread((dense - out)[anchors] * scale): `out` holds the cheap attention of every row, `dense` the full one."""
        seq_len = int(out.shape[0])
        offset = stride - 1 if anchor_offset < 0 else min(anchor_offset, stride - 1)
        anchors = list(range(offset, seq_len, stride))
        if not anchors:
            return
        a_idx = torch.tensor(anchors, dtype=torch.long, device=out.device)
        delta = (dense.index_select(0, a_idx) - out.index_select(0, a_idx)) * scale
        rows, which = self._spread_rows(anchors, seq_len, left=left, right=right, direction=direction)
        out.index_add_(0, torch.tensor(rows, dtype=torch.long, device=out.device),
                       delta.index_select(0, torch.tensor(which, dtype=torch.long, device=out.device)))

    def _sparse_prefill_attention(self, keep: Sequence[torch.Tensor], *, full_prompt_len: int, seq_len: int, delta: bool, stride: int,
                                  left: int, right: int, direction: str, anchor_offset: int, scale: float):
        """The attention of the engine's sparse prefill (reference attention_v4.py:164-289) as a composition of standard calls:
        in layer l every row attends only the keys some KV head keeps in that layer (the union of `keep[l]`) and the MASK slots;
        with `delta`, a second, dense pass gives the exact output at every stride-th row and the difference is spread over the
        rows of that anchor's window. (The reference evaluates the dense pass at the anchor rows only; rows are independent, so
        evaluating it for all rows and reading the anchors gives the same numbers.)"""
        device = self.device

        def attention(layer: int, run, out: torch.Tensor) -> None:
            key_mask = torch.zeros(seq_len, dtype=torch.bool, device=device)
            kept = keep[layer].to(device=device, dtype=torch.long).reshape(-1)
            kept = kept[(kept >= 0) & (kept < seq_len)]
            if kept.numel() == 0:
                run(out)
                return
            key_mask[kept] = True
            key_mask[full_prompt_len:] = True
            run(out, mask=key_mask.unsqueeze(0).expand(seq_len, seq_len).contiguous())
            if delta:
                dense = torch.empty_like(out)
                run(dense)
                self._apply_delta(out, dense, stride=stride, left=left, right=right, direction=direction, anchor_offset=anchor_offset,
                                  scale=scale)

        return attention

    def _decode_with_delta(self, record: DreamPrefillRecord, max_new_tokens: int, stop_token_ids) -> FastDLLMEngineOutput:
        """Block denoising over a compacted prompt with the decode-time delta correction (reference attention_v4.py:86-162): in
        every layer of every step the block rows attend the kept prompt KV as usual, a second pass attends the FULL prompt KV
        (the record's reservoir, loaded into pages of its own for the duration of the decode) plus the block, and the
        difference at every stride-th row is spread over the `left` rows before it. Eager steps (no captured graph)."""
        state = record.decode_delta_state
        page = self.page_size
        full_len = int(state["full_prompt_len"])
        n = int(record.decode_len)
        reservoir: List[int] = []
        try:
            n_pages = math.ceil(full_len / page)
            self._prefix_cache.ensure_free(n_pages)
            reservoir = self._prefix_cache.allocate_pages(n_pages)
            self._load_prompt_cache_per_layer(reservoir, full_len, state["full_k"], state["full_v"])
            m = self.model
            res_table = m.i32(reservoir).view(1, -1)
            res_lens = m.i32([full_len + n])
            stride, left, scale = max(1, int(state.get("stride", 4))), max(0, int(state.get("left", 3))), float(state.get("scale", 1.0))
            anchor_offset = int(state.get("anchor_offset", stride - 1))

            def attention(layer: int, run, out: torch.Tensor) -> None:
                run(out)
                dense = torch.empty_like(out)
                run(dense, block_table=res_table, seq_lens=res_lens, max_seq_len=full_len + n)
                self._apply_delta(out, dense, stride=stride, left=left, right=0, direction="left", anchor_offset=anchor_offset, scale=scale)

            block = torch.full((n,), self.mask_token_id, dtype=torch.long, device=self.device)
            block[0] = int(record.first_token_id)
            slots = slots_for(record.block_page_ids, 0, n, page)
            n_steps, remaining = 0, n - 1
            while remaining > 0:
                n_steps += 1
                if n_steps > n + 8:
                    raise RuntimeError("denoising did not converge: every step must unmask at least one slot")
                logits, _ = self._forward(block, record.suffix_positions, ctx_page_ids=record.prompt_page_ids, ctx_len=record.prompt_len,
                                          store_slots=slots, attention_fn=attention)
                if self._uses_sampler():
                    remaining = self._sampled_unmask(logits, block, record.last_context_logit)
                else:
                    counts = ops.unmask_step(logits, block, mask_token_id=self.mask_token_id, threshold=self.threshold,
                                             last_logit=record.last_context_logit, shift=self.model.arch.logit_shift, softmax_dtype=torch.float32)
                    remaining = int(counts[2].item())
            ops.check_status(self.device)
            return self._finish(block.clone(), max_new_tokens, stop_token_ids, n_steps)
        finally:
            if reservoir:
                self._prefix_cache.release_pages(reservoir)
            self.release_pd_record(record)

    # ------------------------------------------------------------------------------------------------ sampling
    def _uses_sampler(self) -> bool:
        """True when the settings change the greedy fp32-softmax rule that the unmask kernel implements."""
        return self.temperature > 0 or self.top_k is not None or (self.top_p is not None and self.top_p < 1)

    def _sample_tokens(self, logits: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """(confidence, token) per row (reference :1658-1681): fp32 logits over the temperature, top-k filter (what is below the
        k-th largest goes to the floor), THEN the nucleus filter (the smallest sorted prefix whose mass exceeds top_p, its first
        token always kept), softmax; the arg-max and its probability at temperature 0, otherwise one categorical draw from the
        global generator and the drawn token's probability."""
        work = logits.float()
        if self.temperature > 0:
            work = work / self.temperature
        floor = torch.finfo(work.dtype).min
        if self.top_k is not None:
            kth = torch.topk(work, min(int(self.top_k), work.shape[-1]), dim=-1).values[..., -1, None]
            work = work.masked_fill(work < kth, floor)
        if self.top_p is not None and self.top_p < 1:
            ordered, order = torch.sort(work, descending=True, dim=-1)
            drop_sorted = torch.cumsum(F.softmax(ordered, dim=-1), dim=-1) > float(self.top_p)
            drop_sorted[..., 1:] = drop_sorted[..., :-1].clone()
            drop_sorted[..., 0] = False
            drop = torch.zeros_like(work, dtype=torch.bool)
            drop.scatter_(-1, order, drop_sorted)
            work = work.masked_fill(drop, floor)
        probs = F.softmax(work, dim=-1)
        if self.temperature > 0:
            token = torch.distributions.Categorical(probs=probs).sample()
            return torch.gather(probs, -1, token.unsqueeze(-1)).squeeze(-1), token
        return probs.max(dim=-1)

    def _first_token(self, logit_row: torch.Tensor) -> int:
        """The first token of a block from the logit row that predicts it: the arg-max (no filter moves it) or, at a positive
        temperature, a draw."""
        if self.temperature > 0:
            return int(self._sample_tokens(logit_row.reshape(1, -1))[1][0].item())
        return int(torch.argmax(logit_row).item())

    def _sampled_unmask(self, logits: torch.Tensor, block: torch.Tensor, last_logit: Optional[torch.Tensor]) -> int:
        """One confidence-threshold transfer with the sampler's confidences (reference :2143-2157): the masked slots are
        sampled, the most confident one is always accepted and every other one whose confidence reaches the threshold.
        `block` is updated in place; returns the MASK slots left."""
        if self.model.arch.logit_shift:
            shifted = torch.empty_like(logits)
            shifted[1:] = logits[:-1]
            shifted[0] = logits[0] if last_logit is None else last_logit.reshape(-1)
        else:
            shifted = logits
        masked = block == self.mask_token_id
        n_masked = int(masked.sum().item())
        if n_masked == 0:
            return 0
        confidence, sampled = self._sample_tokens(shifted[masked])
        candidate = torch.full_like(block, self.mask_token_id)
        candidate[masked] = sampled
        full_confidence = torch.full(block.shape, -torch.inf, dtype=confidence.dtype, device=block.device)
        full_confidence[masked] = confidence
        best_confidence, best = torch.topk(full_confidence, n_masked)
        accept = torch.zeros_like(block, dtype=torch.bool)
        accept[best[0]] = True
        accept[best[1:][best_confidence[1:] >= self.threshold]] = True
        block[accept] = candidate[accept]
        return int((block == self.mask_token_id).sum().item())

    def _finish(self, block: torch.Tensor, max_new_tokens: int, stop_token_ids, n_steps: int) -> FastDLLMEngineOutput:
        generated = block[:max_new_tokens].tolist()
        if stop_token_ids:
            stop_set = set(int(x) for x in stop_token_ids)
            for idx, token_id in enumerate(generated):
                if token_id in stop_set:
                    generated = generated[:idx]
                    break
        text = ""
        if self.tokenizer is not None:
            text = self.tokenizer.decode(generated, skip_special_tokens=False)
            eos = getattr(self.tokenizer, "eos_token", None)
            if eos and eos in text:
                text = text.split(eos)[0]
        return FastDLLMEngineOutput(text=text, token_ids=generated, n_diff_steps=n_steps)

    @_on_device
    @torch.inference_mode()
    def decode_from_pd_record(self, record: DreamPrefillRecord, *, max_new_tokens: int,
                              stop_token_ids: Optional[Iterable[int]] = None) -> FastDLLMEngineOutput:
        """Denoise the block of a record against its prompt pages; CONSUMES the record (pages released in `finally`,
        reference :2111-2190)."""
        if max_new_tokens <= 0:
            return FastDLLMEngineOutput(text="", token_ids=[], n_diff_steps=0)
        if max_new_tokens > record.decode_len:
            raise ValueError(f"max_new_tokens={max_new_tokens} exceeds record decode_len={record.decode_len}.")
        if record.decode_len > self.block_length:
            return self._decode_blocks(record, max_new_tokens, stop_token_ids)
        if record.decode_delta_state and record.decode_delta_state.get("enabled", False):
            return self._decode_with_delta(record, max_new_tokens, stop_token_ids)
        try:
            block, n_steps = self._denoise_block(
                ctx_page_ids=record.prompt_page_ids, ctx_len=record.prompt_len,
                block_slots=slots_for(record.block_page_ids, 0, record.decode_len, self.page_size),
                block_positions=record.suffix_positions, first_token_id=record.first_token_id,
                last_context_logit=record.last_context_logit)
            ops.check_status(self.device)
            return self._finish(block, max_new_tokens, stop_token_ids, n_steps)
        finally:
            self.release_pd_record(record)

    def _token_run(self, record: DreamPrefillRecord, extra: List[int]) -> _TokenRun:
        """[prompt ‖ suffix] of a record as ONE run of tokens over a page list. The suffix continues in the prompt's last page
        when the record owns its prompt pages; when they belong to the shared prefix cache (other requests read them, and may
        append their own suffix) the partially filled last page is first copied into a private one. Pages allocated here are
        appended to `extra` for the caller to release."""
        page = self.page_size
        n_full, rem = divmod(int(record.prompt_len), page)
        if rem == 0:
            pages = list(record.prompt_page_ids[:n_full]) + list(record.block_page_ids)
        elif record.owns_prompt_pages:
            pages = list(record.prompt_page_ids[:n_full + 1]) + list(record.block_page_ids)
        else:
            private = list(record.block_page_ids)
            need = math.ceil((rem + record.decode_len) / page)
            if need > len(private):
                self._prefix_cache.ensure_free(need - len(private))
                more = self._prefix_cache.allocate_pages(need - len(private))
                extra += more
                private += more
            planes = 2 * int(self.model.kv_cache.shape[1])
            ops.copy_pages(self._layer_pools(), self._all_layer_page_ids([record.prompt_page_ids[n_full]]), self._layer_pools(),
                           self._all_layer_page_ids([private[0]]), n_lists=planes, tokens_per_list=rem)
            pages = list(record.prompt_page_ids[:n_full]) + private
        if len(pages) * page < record.prompt_len + record.decode_len:
            raise RuntimeError("record holds too few pages for its prompt and MASK slots")
        return _TokenRun(pages, int(record.prompt_len), page)

    def _decode_blocks(self, record: DreamPrefillRecord, max_new_tokens: int, stop_token_ids) -> FastDLLMEngineOutput:
        """Several generation blocks on a record (beyond the reference engine, whose first version stops at one block:
        fastdllm_engine.py:1911-1915, 2286-2290). The block loop is the eval class's dual cache (fastdllm_parallelcomp.py
        :2932-2998) with the engine's fp32 softmax: every block starts by forwarding all remaining MASK slots against
        [prompt ‖ finished blocks], the active block's rows replace their slots at every step and see the later MASK slots,
        a commit forward stores the finished block. Only the prompt KV crosses the prefill/decode boundary: the MASK slots
        are recomputed here, so a record that came from a snapshot or from another engine decodes the same way.
        The loop needs [prompt ‖ suffix] as ONE run of tokens over a page list. The suffix continues in the prompt's last
        page when the record owns its prompt pages; when they belong to the shared prefix cache (other requests read them, and
        may append their own suffix) the partially filled last page is first copied into a private one."""
        extra: List[int] = []
        try:
            view = self._token_run(record, extra)
            steps: List[int] = []
            generated = denoise_blocks(self.model, view, suffix_pos_start=int(record.suffix_positions[0]), last_logit=record.last_context_logit,
                                       first_token=None, tail_in_cache=0, max_new=int(max_new_tokens), block_length=self.block_length,
                                       mask_id=self.mask_token_id, threshold=self.threshold, softmax_dtype=torch.float32,
                                       use_graph=not self.config.enforce_eager, steps_out=steps,
                                       pick_first_token=(lambda row: torch.tensor(self._first_token(row), device=self.device)) if self.temperature > 0 else None,
                                       threshold_step=self._sampled_unmask if self._uses_sampler() else None)
            ops.check_status(self.device)
            block = torch.tensor(generated, dtype=torch.long)
            return self._finish(block, max_new_tokens, stop_token_ids, sum(steps))
        finally:
            if extra:
                self._prefix_cache.release_pages(extra)
            self.release_pd_record(record)

    @_on_device
    @torch.inference_mode()
    def decode_from_pd_records(self, records: Sequence[DreamPrefillRecord], *, max_new_tokens: int,
                               stop_token_ids: Optional[Iterable[int]] = None) -> List[FastDLLMEngineOutput]:
        """Denoise the blocks of SEVERAL records in shared steps: their rows are packed into one forward per step (each
        against its own prompt pages), so the model's weights are read once per step for all of them instead of once
        per request. Same result per request as `decode_from_pd_record`; consumes every record. Not in the reference
        facade, whose decode loop serves one request (its batching lives in the scheduler of the underlying engine)."""
        records = list(records)
        if not records:
            return []
        if max_new_tokens <= 0:
            return [FastDLLMEngineOutput(text="", token_ids=[], n_diff_steps=0) for _ in records]
        decode_len = records[0].decode_len
        if self._uses_sampler() or any(r.decode_delta_state and r.decode_delta_state.get("enabled", False) for r in records):
            # the delta correction runs a second attention pass per record, and a sampler runs eager steps: one record after the other
            return [self.decode_from_pd_record(r, max_new_tokens=max_new_tokens, stop_token_ids=stop_token_ids) for r in records]
        try:
            for r in records:
                if r.decode_len != decode_len:
                    raise ValueError("records of one batch must share decode_len")
                if max_new_tokens > r.decode_len:
                    raise ValueError(f"max_new_tokens={max_new_tokens} exceeds record decode_len={r.decode_len}.")
            if decode_len > self.block_length:
                return self._decode_blocks_shared(records, int(max_new_tokens), stop_token_ids)
            requests = [dict(positions=r.suffix_positions, ctx_page_ids=r.prompt_page_ids, ctx_len=r.prompt_len,
                             last_logit=r.last_context_logit, store_slots=slots_for(r.block_page_ids, 0, decode_len, self.page_size))
                        for r in records]
            runner = self.model.batched_step_runner(block_len=decode_len, requests=requests, mask_token_id=self.mask_token_id,
                                                    threshold=self.threshold, shift=self.model.arch.logit_shift, softmax_dtype=torch.float32,
                                                    use_graph=not self.config.enforce_eager)
            for block, r in zip(runner.blocks, records):
                block.fill_(self.mask_token_id)
                block[0] = int(r.first_token_id)
            steps_needed = [0] * len(records)
            step, left = 0, [decode_len - 1] * len(records)
            while any(x > 0 for x in left):
                step += 1
                runner.run()
                for i, (before, after) in enumerate(zip(left, runner.remaining)):
                    if before > 0 and after == 0:
                        steps_needed[i] = step
                left = list(runner.remaining)
                if step > decode_len + 8:
                    raise RuntimeError("denoising did not converge: every step must unmask at least one slot")
            ops.check_status(self.device)
            return [self._finish(block.clone(), max_new_tokens, stop_token_ids, steps_needed[i]) for i, block in enumerate(runner.blocks)]
        finally:
            for r in records:
                self.release_pd_record(r)

    def _decode_blocks_shared(self, records: List[DreamPrefillRecord], max_new_tokens: int, stop_token_ids) -> List[FastDLLMEngineOutput]:
        """Records of several blocks in shared steps: the dual-cache block loop of `_decode_blocks`, every forward of it packed over
        the records (`model.denoise_blocks_batched`). The caller releases the records."""
        extra: List[int] = []
        try:
            views = [self._token_run(r, extra) for r in records]
            steps: List[List[int]] = [[] for _ in records]
            generated = denoise_blocks_batched(self.model, views, suffix_pos_starts=[int(r.suffix_positions[0]) for r in records],
                                               last_logits=[r.last_context_logit for r in records], max_new=max_new_tokens,
                                               block_length=self.block_length, mask_id=self.mask_token_id, threshold=self.threshold,
                                               softmax_dtype=torch.float32, use_graph=not self.config.enforce_eager, steps_out=steps)
            ops.check_status(self.device)
            return [self._finish(torch.tensor(g, dtype=torch.long), max_new_tokens, stop_token_ids, sum(st)) for g, st in zip(generated, steps)]
        finally:
            if extra:
                self._prefix_cache.release_pages(extra)

    def _require_shifted_logits(self, what: str) -> None:
        """The selection / chunk-local twins restate Dream's shifted read-out only (the reference engine has no other model)."""
        if not self.model.arch.logit_shift:
            raise NotImplementedError(f"{what} is built for architectures with shifted logits (Dream) only")

    def release_pd_record(self, record: DreamPrefillRecord) -> None:
        """Release the pages of a record that will not be decoded (reference :2192-2198)."""
        self._prefix_cache.release_pages(record.block_page_ids)
        if record.owns_prompt_pages:
            self._prefix_cache.release_pages(record.prompt_page_ids)
        if record.cached_prefix is not None:
            record.cached_prefix.ref_count -= 1

    @torch.inference_mode()
    def generate_token_ids_pd_split(self, prompt_ids: Sequence[int], *, max_new_tokens: int, stop_token_ids: Optional[Iterable[int]] = None,
                                    **prefill_kwargs) -> FastDLLMEngineOutput:
        """Prefill then decode through the explicit boundary (reference :2201-2255)."""
        record = self.prefill_to_pd_record(prompt_ids, max_new_tokens=max_new_tokens, **prefill_kwargs)
        return self.decode_from_pd_record(record, max_new_tokens=max_new_tokens, stop_token_ids=stop_token_ids)

    @torch.inference_mode()
    def generate_token_ids(self, prompt_ids: Sequence[int], *, max_new_tokens: int, stop_token_ids: Optional[Iterable[int]] = None,
                           **prefill_kwargs) -> FastDLLMEngineOutput:
        """Same result as the PD split; the reference keeps a fused copy of the two halves (:2258-2528)."""
        if max_new_tokens <= 0:
            return FastDLLMEngineOutput(text="", token_ids=[], n_diff_steps=0)
        return self.generate_token_ids_pd_split(prompt_ids, max_new_tokens=max_new_tokens, stop_token_ids=stop_token_ids, **prefill_kwargs)

    def generate(self, prompts, sampling_params) -> List[FastDLLMEngineOutput]:
        """`sampling_params`: any object with `max_tokens` and `stop_token_ids` (list of lists), reference :2530-2556."""
        stop_token_ids = None
        if getattr(sampling_params, "stop_token_ids", None):
            stop_token_ids = [item for group in sampling_params.stop_token_ids for item in group]
        outputs = []
        for prompt in prompts:
            if isinstance(prompt, str):
                if self.tokenizer is None:
                    raise ValueError("text prompts need a tokenizer in the checkpoint directory")
                prompt_ids = self.tokenizer.encode(prompt)
            else:
                prompt_ids = list(prompt)
            outputs.append(self.generate_token_ids(prompt_ids, max_new_tokens=int(sampling_params.max_tokens), stop_token_ids=stop_token_ids))
        return outputs

    # ------------------------------------------------------------------------------------------------ chunk selection
    @staticmethod
    def _select_attention_layer_indices(total_layers: int, layer_window: int, layer_mode: str) -> List[int]:
        """Layers whose attention is scored: all of them, or a window of `layer_window` at either end."""
        every = list(range(max(0, total_layers)))
        if not every or layer_mode == "all" or layer_window <= 0:
            return every
        if layer_mode not in ("first", "last"):
            raise ValueError(f"Unsupported attention layer mode: {layer_mode}")
        width = min(max(1, int(layer_window)), total_layers)
        return every[:width] if layer_mode == "first" else every[-width:]

    @staticmethod
    def _window_query(query_ids: Sequence[int], window: int) -> List[int]:
        ids = [int(x) for x in query_ids]
        return ids[-int(window):] if window and window > 0 else ids

    @_on_device
    @torch.inference_mode()
    def generate_partial_draft_rounds_for_selection(self, prompt_ids: Sequence[int], *, max_new_tokens: int,
                                                    partial_rounds: int) -> Tuple[List[int], List[bool]]:
        """Engine draft (reference :1014-1060): every round is ONE bidirectional forward over `[prompt ‖ draft block]`
        with nothing cached (prompt rows see the MASK slots — unlike the eval class, which drafts against a cached
        prompt). Slot 0 comes from the last prompt row; each further round confirms the most confident masked slot."""
        draft_len = int(max_new_tokens or 0)
        if draft_len <= 0:
            return [], []
        self._require_shifted_logits("generate_partial_draft_rounds_for_selection")
        prompt_ids = [int(x) for x in prompt_ids]
        p_len = len(prompt_ids)
        if p_len <= 0:
            raise ValueError("the draft needs at least one prompt token")
        positions = list(range(p_len + draft_len))
        block = torch.full((draft_len,), self.mask_token_id, dtype=torch.long, device=self.device)
        prompt_t = self.model.ids_tensor(prompt_ids)
        rows = list(range(p_len - 1, p_len + draft_len - 1))        # shifted: slot j reads the logits of row p_len + j - 1
        logits, _ = self._forward(torch.cat([prompt_t, block]), positions, logit_rows=rows[:1])
        block[0] = self._first_token(logits[0])
        confirmed = torch.zeros(draft_len, dtype=torch.bool, device=self.device)
        confirmed[0] = True
        for _ in range(max(0, int(partial_rounds or 0))):
            if not bool((block == self.mask_token_id).any()):
                break
            before = block.clone()
            logits, _ = self._forward(torch.cat([prompt_t, block]), positions, logit_rows=rows)
            if self._uses_sampler():
                # the most confident masked slot by the sampler's confidences takes its sampled token (reference :1053-1059)
                masked = (block == self.mask_token_id).nonzero(as_tuple=True)[0]
                confidence, sampled = self._sample_tokens(logits.index_select(0, masked))
                best = int(torch.argmax(confidence).item())
                block[masked[best]] = sampled[best]
                confirmed[masked[best]] = True
                continue
            with torch.cuda.device(self.device):
                # rows are already the shifted ones; a threshold no probability reaches leaves only the top-1 transfer
                ops.unmask_step(logits, block, mask_token_id=self.mask_token_id, threshold=2.0, shift=False, softmax_dtype=torch.float32)
            confirmed |= block != before
        return block.tolist(), confirmed.tolist()

    def _selection_query_ids_with_score_target_engine(self, prefix_ids, scoring_query_ids, *, score_mode: str, score_draft_tokens: int = 0,
                                                      score_draft_partial_rounds: Optional[int] = None,
                                                      score_draft_score_all_slots: bool = False):
        selection = [int(x) for x in scoring_query_ids]
        mask: Optional[List[bool]] = None
        if (score_mode or "").lower() == "draft_self_information" and int(score_draft_tokens or 0) > 0:
            if score_draft_partial_rounds is not None:
                draft_ids, draft_mask = self.generate_partial_draft_rounds_for_selection(
                    list(prefix_ids) + list(scoring_query_ids), max_new_tokens=int(score_draft_tokens),
                    partial_rounds=int(score_draft_partial_rounds))
                mask = [True] * len(scoring_query_ids) + ([True] * len(draft_ids) if score_draft_score_all_slots else list(draft_mask))
            else:
                draft_ids = list(self.generate_token_ids(list(prefix_ids) + list(scoring_query_ids),
                                                         max_new_tokens=int(score_draft_tokens), stop_token_ids=None).token_ids)
            selection = list(scoring_query_ids) + list(draft_ids)
        return selection, None, mask

    @staticmethod
    def _label_positions(prefix_len: int, chunk_len: int, query_ids: Sequence[int], score_token_count, score_token_mask):
        """(label positions, label ids) of one scoring row, or None when the row scores -inf (reference :1118-1140)."""
        query_len = len(query_ids)
        start = prefix_len + chunk_len
        if score_token_mask is not None:
            if len(score_token_mask) != query_len:
                return None
            local = [i for i, keep in enumerate(score_token_mask) if keep]
            if not local:
                return None
            positions, labels = [start + i for i in local], [query_ids[i] for i in local]
        elif score_token_count is None:
            positions, labels = list(range(start, start + query_len)), list(query_ids)
        else:
            target = min(query_len, max(0, int(score_token_count)))
            if target <= 0:
                return None
            positions, labels = list(range(start, start + target)), list(query_ids[:target])
        if not positions or min(positions) <= 0:
            return None
        return positions, labels

    @_on_device
    @torch.inference_mode()
    def score_chunk_self_information_engine(self, prefix_ids, chunk_ids, query_ids, *, score_token_count: Optional[int] = None,
                                            score_token_mask: Optional[Sequence[bool]] = None, score_attention_mask: str = "causal") -> float:
        """mean log p(label | prefix, chunk, earlier query) of one chunk (reference :1097-1152); LM head on label rows only."""
        prefix_ids, chunk_ids, query_ids = [int(x) for x in prefix_ids], [int(x) for x in chunk_ids], [int(x) for x in query_ids]
        if not chunk_ids or not query_ids:
            return float("-inf")
        target = self._label_positions(len(prefix_ids), len(chunk_ids), query_ids, score_token_count, score_token_mask)
        if target is None:
            return float("-inf")
        positions, labels = target
        joint = prefix_ids + chunk_ids + query_ids
        causal, mask = self._selection_mask(score_attention_mask, seq_len=len(joint), prefix_len=len(prefix_ids),
                                            chunk_len=len(chunk_ids), query_len=len(query_ids))
        logits, _ = self._forward(joint, list(range(len(joint))), causal=causal, mask=mask, logit_rows=[p - 1 for p in positions])
        with torch.cuda.device(self.device):
            score = float(ops.self_information_scores(logits, self.model.ids_tensor(labels), 1)[0].item())
        return score if math.isfinite(score) else float("-inf")

    @_on_device
    @torch.inference_mode()
    def select_chunks_by_engine(self, prefix_ids, candidate_chunks, scoring_query_ids, *, topk_chunks: int,
                                score_mode: str = "draft_self_information", score_draft_tokens: int = 4,
                                score_draft_partial_rounds: Optional[int] = 1, score_draft_score_all_slots: bool = False,
                                score_attention_mask: str = "causal", score_context_mode: str = "single_chunk",
                                keep_first_chunk: bool = False, score_batch_size: int = 8):
        """(selected ascending, scores, selection query ids, label mask) — reference :1154-1204. Chunks of equal length are
        scored `score_batch_size` at a time in one packed forward (the reference forwards one chunk at a time); the
        ranking is the stable descending sort of the reference, run by the top-K kernel."""
        if not candidate_chunks:
            return [], {}, list(scoring_query_ids), None
        selection, count, mask = self._selection_query_ids_with_score_target_engine(
            prefix_ids, scoring_query_ids, score_mode=score_mode, score_draft_tokens=score_draft_tokens,
            score_draft_partial_rounds=score_draft_partial_rounds, score_draft_score_all_slots=score_draft_score_all_slots)
        if (score_mode or "none").lower() == "none" or not selection:
            selected = list(range(len(candidate_chunks)))
            if int(topk_chunks or 0) > 0:
                selected = selected[:int(topk_chunks)]
            return selected, {}, selection, mask
        if score_context_mode != "single_chunk":
            raise ValueError(f"Engine chunk selection currently supports score_context_mode='single_chunk', got {score_context_mode!r}.")
        if (score_mode or "").lower() not in {"self_information", "draft_self_information"}:
            raise ValueError(f"Engine chunk selection currently supports self_information/draft_self_information, got {score_mode!r}.")
        scores = self._score_chunks_batched([int(x) for x in prefix_ids], candidate_chunks, selection, count, mask,
                                            score_attention_mask, max(1, int(score_batch_size or 1)))
        dense = torch.tensor([scores[i] for i in range(len(candidate_chunks))], dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            sel, cnt = ops.topk_chunks(dense, int(topk_chunks or 0), bool(keep_first_chunk))
        return sel[: int(cnt.item())].tolist(), scores, selection, mask

    def _score_chunks_batched(self, prefix_ids, candidate_chunks, query_ids, count, mask, attention_mask: str, batch_size: int) -> Dict[int, float]:
        m = self.model
        scores: Dict[int, float] = {}
        groups: Dict[int, List[Tuple[int, List[int]]]] = {}
        for idx, chunk in enumerate(candidate_chunks):
            chunk = [int(x) for x in chunk]
            if not chunk or not query_ids:
                scores[idx] = float("-inf")
            else:
                groups.setdefault(len(chunk), []).append((idx, chunk))
        mode = (attention_mask or "full").lower()
        for c_len, group in groups.items():
            target = self._label_positions(len(prefix_ids), c_len, query_ids, count, mask)
            if target is None:
                scores.update({idx: float("-inf") for idx, _ in group})
                continue
            positions, labels = target
            if mode == "query_to_chunk":   # needs a dense mask, which is per sequence: one chunk per forward
                for idx, chunk in group:
                    scores[idx] = self.score_chunk_self_information_engine(prefix_ids, chunk, query_ids, score_token_count=count,
                                                                           score_token_mask=mask, score_attention_mask=attention_mask)
                continue
            causal, _ = self._selection_mask(mode, seq_len=0, prefix_len=0, chunk_len=0, query_len=0)
            row_len = len(prefix_ids) + c_len + len(query_ids)
            labels_t = m.ids_tensor(labels)
            for off in range(0, len(group), batch_size):
                batch = group[off:off + batch_size]
                flat = [t for _, chunk in batch for t in (prefix_ids + chunk + list(query_ids))]
                cu = [b * row_len for b in range(len(batch) + 1)]
                rows = [b * row_len + (p - 1) for b in range(len(batch)) for p in positions]
                with torch.cuda.device(self.device):
                    logits, _ = m.forward(m.ids_tensor(flat), torch.arange(row_len, device=m.device).repeat(len(batch)),
                                          cu_seqlens=m.i32(cu), max_query_len=row_len, causal=causal, logit_rows=m.ids_tensor(rows))
                    vals = ops.self_information_scores(logits, labels_t, len(batch)).tolist()
                for (idx, _), v in zip(batch, vals):
                    scores[idx] = v if math.isfinite(v) else float("-inf")
        return scores

    # ------------------------------------------------------------------------------------------------ token eviction
    @_on_device
    @torch.inference_mode()
    def compute_prompt_keep_indices_per_layer_per_head(self, *, full_prompt_len: int, prefix_ids, chunk_spans, query_ids, token_capacity: int,
                                                       token_score_query_window: int = 8, token_score_layers: int = 1,
                                                       token_score_layer_mode: str = "first", token_score_reduce: str = "sum",
                                                       token_score_pooling: str = "maxpool", token_score_pool_kernel: int = 7,
                                                       token_score_direction: str = "query_to_chunk", token_score_keep: str = "high",
                                                       token_score_include_prefix: bool = True, token_attention_mask: str = "causal",
                                                       token_score_backend: str = "torch", return_selection_dense_outputs: bool = False):
        """Per layer and KV head, which prompt tokens stay (reference :1325-1563).

        `chunk_spans`: dicts with `chunk_ids`, `start`, `end` (span of the chunk inside the full prompt). For a chunk
        longer than `token_capacity`: one bidirectional forward over `[prefix ‖ chunk ‖ query window]` with nothing
        stored, the rotated q / k of the selected layers go to the fused scorer (query→chunk attention mass under
        `token_attention_mask`; with `token_score_direction` "chunk_to_query" / "bidirectional" also the mass the chunk rows put
        on the window), then max / average / no pooling, mean over each KV head's query heads, BOS + top-(capacity - 1) (or the
        lowest, `token_score_keep="low"`), ascending.
        Returns (keep `[layers][Hkv][active_len]` as nested lists, per-chunk meta). `token_score_backend` is accepted for
        signature parity: there is one backend."""
        if return_selection_dense_outputs:
            raise NotImplementedError("selection dense outputs (for the sparse delta prefill) are not built")
        direction = (token_score_direction or "query_to_chunk").lower()
        if direction not in {"query_to_chunk", "chunk_to_query", "bidirectional"}:
            raise ValueError(f"Unsupported token_score_direction: {token_score_direction}")
        pooling = (token_score_pooling or "none").lower()
        if pooling not in {"none", "maxpool", "avgpool"}:
            raise ValueError(f"Unsupported token_score_pooling: {token_score_pooling}")
        # the selection kernel max-pools; average pooling is applied to the head scores beforehand (torch), the kernel then pools over 1
        pool_kernel = int(token_score_pool_kernel or 1) if pooling == "maxpool" else 1
        capacity = int(token_capacity or 0)
        query_ids = self._window_query(query_ids, token_score_query_window)
        arch = self.model.arch
        num_layers, hkv = arch.num_hidden_layers, arch.num_key_value_heads
        selected_layers = self._select_attention_layer_indices(num_layers, token_score_layers, token_score_layer_mode) or [0]
        all_layer_keeps: List[List[torch.Tensor]] = [[] for _ in range(num_layers)]
        chunk_meta: List[Dict[str, int]] = []
        for span in chunk_spans:
            chunk_ids = [int(x) for x in span["chunk_ids"]]
            start, end = int(span["start"]), int(span["end"])
            chunk_len = len(chunk_ids)
            keep_count = min(max(1, capacity), chunk_len) if capacity > 0 else chunk_len
            if chunk_len <= 0:
                chunk_meta.append({"start": start, "end": end, "kept_tokens": 0, "union_kept_tokens": 0})
                continue
            if capacity <= 0 or chunk_len <= capacity or not query_ids:
                base = torch.arange(chunk_len, device=self.device, dtype=torch.long)
                per_layer_keep = [base.unsqueeze(0).expand(hkv, -1).clone() for _ in range(num_layers)]
            else:
                prefix = [int(x) for x in prefix_ids] if token_score_include_prefix else []
                joint = prefix + chunk_ids + list(query_ids)
                # the hidden states run under FULL attention; only the score softmax applies `token_attention_mask`
                _, captured = self._forward(joint, list(range(len(joint))), want_logits=False, capture_layers=selected_layers)
                with torch.cuda.device(self.device):
                    head_scores = torch.stack([
                        self._chunk_head_scores(captured[l][0], captured[l][1], prefix_len=len(prefix), chunk_len=chunk_len, query_len=len(query_ids),
                                                direction=direction, reduce_mode=token_score_reduce, attention_mask=token_attention_mask)
                        for l in selected_layers], dim=0).contiguous()
                    if pooling == "avgpool":
                        kernel = max(1, min(int(token_score_pool_kernel or 1), chunk_len))
                        flat = head_scores.reshape(-1, 1, chunk_len)
                        head_scores = F.avg_pool1d(flat, kernel_size=kernel, padding=kernel // 2, stride=1)[..., :chunk_len].reshape(head_scores.shape).contiguous()
                    keeps = ops.evict_select(head_scores, num_kv_heads=hkv, keep_count=keep_count, pool_kernel=pool_kernel, per_head=True,
                                             force_keep_first=True, keep_high=token_score_keep == "high")
                per_layer_keep = [keeps[min(layer_idx, len(selected_layers) - 1)].clone() for layer_idx in range(num_layers)]
            union = torch.unique(torch.cat([k.reshape(-1) for k in per_layer_keep]))
            for layer_idx, layer_keep in enumerate(per_layer_keep):
                all_layer_keeps[layer_idx].append(layer_keep + start)
            chunk_meta.append({"start": start, "end": end, "kept_tokens": keep_count, "union_kept_tokens": int(union.numel())})

        spans_with_keep = [s for s in chunk_spans if len(s["chunk_ids"]) > 0]
        prompt_keep: List[List[List[int]]] = []
        for layer_idx, layer_parts in enumerate(all_layer_keeps):
            if not layer_parts:
                base = torch.arange(full_prompt_len, device=self.device, dtype=torch.long)
                prompt_keep.append(base.unsqueeze(0).expand(hkv, -1).tolist())
                continue
            heads = []
            for head_idx in range(int(layer_parts[0].shape[0])):
                pieces, cursor = [], 0
                for span, layer_keep in zip(spans_with_keep, layer_parts):
                    start, end = int(span["start"]), int(span["end"])
                    if start > cursor:
                        pieces.append(torch.arange(cursor, start, device=self.device, dtype=torch.long))
                    pieces.append(layer_keep[head_idx])
                    cursor = end
                if cursor < full_prompt_len:
                    pieces.append(torch.arange(cursor, full_prompt_len, device=self.device, dtype=torch.long))
                heads.append(torch.cat(pieces, dim=0))
            prompt_keep.append(torch.stack(heads, dim=0).tolist())
        ops.check_status(self.device)
        return prompt_keep, chunk_meta

    def _chunk_head_scores(self, q: torch.Tensor, k: torch.Tensor, *, prefix_len: int, chunk_len: int, query_len: int, direction: str,
                           reduce_mode: str, attention_mask: str) -> torch.Tensor:
        """fp32 [Hq, chunk_len] (reference _engine_chunk_attention_head_scores :1230-1323): the attention mass the query window's
        rows put on each chunk token (the fused scorer), and / or the mass each chunk row puts on the query window's keys — that
        one on torch ops: a softmax over all keys of the chunk rows, under the score mask (zero under the causal and
        query_to_chunk masks, where chunk rows do not see the query)."""
        parts = []
        if direction in {"query_to_chunk", "bidirectional"}:
            parts.append(ops.query_to_chunk_attention_scores(q, k, prefix_len=prefix_len, chunk_len=chunk_len, query_len=query_len,
                                                             scale=self.model.scale, reduce_mode=reduce_mode, attention_mask=attention_mask))
        if direction in {"chunk_to_query", "bidirectional"}:
            hq, hkv = int(q.shape[1]), int(k.shape[1])
            if (attention_mask or "full").lower() in {"full", "none"}:
                rows = q[prefix_len:prefix_len + chunk_len].float().transpose(0, 1)                       # [Hq, C, D]
                keys = k.float().transpose(0, 1).repeat_interleave(hq // hkv, dim=0)                      # [Hq, L, D]
                prob = torch.softmax(torch.matmul(rows, keys.transpose(1, 2)) * self.model.scale, dim=-1)
                mass = prob[:, :, prefix_len + chunk_len:prefix_len + chunk_len + query_len]
                parts.append(mass.mean(dim=2) if reduce_mode == "mean" else mass.sum(dim=2))
            elif (attention_mask or "").lower() in {"causal", "query_to_chunk"}:
                parts.append(torch.zeros((hq, chunk_len), dtype=torch.float32, device=q.device))
            else:
                raise ValueError(f"Unsupported token attention mask: {attention_mask}")
        return parts[0] if len(parts) == 1 else parts[0] + parts[1]

    # ------------------------------------------------------------------------------------------------ chunk-local KV
    @_on_device
    @torch.inference_mode()
    def generate_token_ids_from_chunk_local_kv(self, *, prefix_ids, prefix_positions, chunk_ids_list, chunk_positions_list,
                                               chunk_keep_indices_per_layer_per_head, query_ids, query_positions,
                                               local_query_ids: Optional[Sequence[int]] = None, local_attention_mask: str = "causal",
                                               max_new_tokens: int, stop_token_ids: Optional[Iterable[int]] = None) -> FastDLLMEngineOutput:
        """Generate from independently prefilled chunks (reference :1683-1876): every chunk is forwarded as
        `[prefix ‖ chunk ‖ local query]` into scratch pages, its kept tokens are copied per layer and KV head behind the
        prefix in the prompt pages, then `[query ‖ MASK block]` is appended and the block is denoised."""
        if max_new_tokens <= 0:
            return FastDLLMEngineOutput(text="", token_ids=[], n_diff_steps=0)
        if max_new_tokens > self.block_length:
            raise NotImplementedError("FastDLLMDreamEngine chunk-local KV path supports one generation block only. "
                                      f"Got max_new_tokens={max_new_tokens}, block_length={self.block_length}.")
        self._require_shifted_logits("generate_token_ids_from_chunk_local_kv")
        prefix_ids, prefix_positions = [int(x) for x in prefix_ids], [int(x) for x in prefix_positions]
        query_ids, query_positions = [int(x) for x in query_ids], [int(x) for x in query_positions]
        if len(prefix_ids) != len(prefix_positions):
            raise ValueError("prefix_ids/prefix_positions length mismatch")
        if len(query_ids) != len(query_positions):
            raise ValueError("query_ids/query_positions length mismatch")
        if len(chunk_ids_list) != len(chunk_positions_list):
            raise ValueError("chunk ids/positions list length mismatch")
        if len(chunk_ids_list) != len(chunk_keep_indices_per_layer_per_head):
            raise ValueError("chunk ids/keep-indices list length mismatch")
        decode_len = self.block_length
        local_query_ids = [int(x) for x in (local_query_ids if local_query_ids is not None else query_ids)]
        keeps: List[List[torch.Tensor]] = []
        kept_counts: List[int] = []
        for chunk_ids, chunk_keep in zip(chunk_ids_list, chunk_keep_indices_per_layer_per_head):
            tensors, active_len = self._normalize_per_head_keep_indices(chunk_keep, full_prompt_len=len(chunk_ids))
            keeps.append(tensors)
            kept_counts.append(active_len)
        p_len = len(prefix_ids)
        base_len = p_len + sum(kept_counts)
        prompt_len = base_len + len(query_ids)
        suffix_start = (max(query_positions) + 1) if query_positions else (max(prefix_positions) + 1 if prefix_positions else 0)
        block_positions = list(range(suffix_start, suffix_start + decode_len))
        total_slots = prompt_len + decode_len
        if total_slots > self.config.max_model_len:
            raise ValueError(f"chunk-local KV prompt length {total_slots} exceeds max_model_len={self.config.max_model_len}")
        total_pages = math.ceil(total_slots / self.page_size)
        self._prefix_cache.ensure_free(total_pages)
        all_pages = self._prefix_cache.allocate_pages(total_pages)
        scratch: List[int] = []
        try:
            if prefix_ids:
                self._forward(prefix_ids, prefix_positions, store_slots=slots_for(all_pages, 0, p_len, self.page_size), want_logits=False)
            dst = p_len
            for chunk_ids_raw, chunk_pos_raw, chunk_keep in zip(chunk_ids_list, chunk_positions_list, keeps):
                chunk_ids, chunk_pos = [int(x) for x in chunk_ids_raw], [int(x) for x in chunk_pos_raw]
                if len(chunk_ids) != len(chunk_pos):
                    raise ValueError("chunk ids/positions length mismatch")
                if not chunk_ids:
                    continue
                lq_start = max(chunk_pos) + 1
                local_ids = prefix_ids + chunk_ids + local_query_ids
                local_pos = prefix_positions + chunk_pos + list(range(lq_start, lq_start + len(local_query_ids)))
                n_scratch = math.ceil(len(local_ids) / self.page_size)
                self._prefix_cache.ensure_free(n_scratch)
                scratch = self._prefix_cache.allocate_pages(n_scratch)
                causal, mask = self._selection_mask(local_attention_mask, seq_len=len(local_ids), prefix_len=p_len,
                                                    chunk_len=len(chunk_ids), query_len=len(local_query_ids))
                self._forward(local_ids, local_pos, store_slots=slots_for(scratch, 0, len(local_ids), self.page_size), causal=causal,
                              mask=mask, want_logits=False)
                dst += self._copy_chunk_local_kv_to_prompt_pages(src_page_ids=scratch, dst_page_ids=all_pages, src_chunk_start=p_len,
                                                                 dst_start=dst, keep_indices_per_layer_per_head=chunk_keep)
                self._prefix_cache.release_pages(scratch)
                scratch = []
            if dst != base_len:
                raise ValueError(f"chunk-local KV base length mismatch: {dst} vs {base_len}")
            # [query ‖ MASK block] appended behind the compacted base; the reference pads this forward to a multiple of the
            # block length and hides the padding from the valid rows, so the padding is simply not forwarded here
            suffix_ids = query_ids + [self.mask_token_id] * decode_len
            q_len = len(query_ids)
            if q_len <= 0:
                raise ValueError("generate_token_ids_from_chunk_local_kv needs a non-empty query")
            logits, _ = self._forward(suffix_ids, query_positions + block_positions, ctx_page_ids=all_pages, ctx_len=base_len,
                                      store_slots=slots_for(all_pages, base_len, len(suffix_ids), self.page_size), logit_rows=[q_len - 1])
            last_context_logit = logits[0].detach()
            first_token = self._first_token(last_context_logit)
            block, n_steps = self._denoise_block(ctx_page_ids=all_pages, ctx_len=prompt_len,
                                                 block_slots=slots_for(all_pages, prompt_len, decode_len, self.page_size),
                                                 block_positions=block_positions, first_token_id=first_token,
                                                 last_context_logit=last_context_logit)
            ops.check_status(self.device)
        finally:
            if scratch:
                self._prefix_cache.release_pages(scratch)
            self._prefix_cache.release_pages(all_pages)
        return self._finish(block, max_new_tokens, stop_token_ids, n_steps)
