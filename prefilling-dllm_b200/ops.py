"""Op table of the hot path, with the names and signatures of the reference's Python ops.

Reference op table: prefilling_dllm_engine/prefilling_dllm/layers/attention/ops/__init__.py:1-6 and
.../ops/triton_eviction_scorer.py:114. Every function here validates like the reference does (same
exception types), then calls one entry point of libpdllm_b200.so on torch's current CUDA stream.
Tensors stay where they are: the ops write in place and never synchronise.
"""

from __future__ import annotations

import ctypes
import math
import threading
from typing import Dict, Optional, Tuple

import torch

from . import _lib
from ._lib import AttnParams

# Calls made into the C-ABI (every one enqueues at least one kernel); a replayed CUDA graph adds the calls it captured.
# Read by benchmarks that report how many launches a timed region made.
C_ABI_CALLS = 0


def check(code: int) -> None:
    global C_ABI_CALLS
    C_ABI_CALLS += 1
    _lib.check(code)


_DTYPE_CODE = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}; expected float32, bfloat16 or float16") from None


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("pdllm_b200 ops require CUDA tensors (there is no CPU path)")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError(f"tensors live on different devices: {device} vs {t.device}")
    if device is None:
        raise ValueError("no tensor given")
    return device


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


class _DeviceState(threading.local):
    """Per-thread, per-device scratch: the status word and grow-only workspaces."""

    def __init__(self) -> None:
        self.status: Dict[torch.device, torch.Tensor] = {}
        self.workspaces: Dict[Tuple[torch.device, str], torch.Tensor] = {}
        self.graph_held: set = set()      # workspaces whose pointer a captured CUDA graph holds
        self.retired: list = []           # replaced workspaces that such a graph may still use: kept alive


_state = _DeviceState()


def status_word(device: torch.device) -> torch.Tensor:
    word = _state.status.get(device)
    if word is None:
        with torch.inference_mode(False):   # long-lived and reset in place later: must not be an inference tensor
            word = torch.zeros(1, dtype=torch.int32, device=device)
        _state.status[device] = word
    return word


def check_status(device: Optional[torch.device] = None, *, reset: bool = True) -> int:
    """Read the device status word (this synchronises) and raise if a kernel flagged bad input."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    word = status_word(torch.device(device))
    code = int(word.item())
    if code != 0 and reset:
        word.zero_()
    if (code & 0xff) == _lib.S_WAIT_TIMEOUT:
        # an abandoned attention launch may have left split-KV arrival counters behind in the workspace header
        for key in ("attn", "linear"):
            ws = _state.workspaces.get((torch.device(device), key))
            if ws is not None:
                ws[: 64 * 1024].zero_()
    if code != 0:
        detail = f" (barrier {(code >> 8) & 0xff}, warp {(code >> 16) & 0xff}, parity {(code >> 24) & 1})" if code > 0xff else ""
        raise RuntimeError(f"pdllm_b200 device status {code & 0xff}: {_lib.STATUS_NAMES.get(code & 0xff, 'unknown')}{detail}")
    return code


def _workspace(device: torch.device, key: str, nbytes: int, *, zero: bool = False) -> torch.Tensor:
    """Grow-only scratch per (thread, device, key). Launches that share a buffer must be ordered on one stream."""
    capturing = torch.cuda.is_current_stream_capturing()
    buf = _state.workspaces.get((device, key))
    if buf is not None and buf.numel() >= nbytes:
        if capturing:
            # A captured launch keeps this pointer for as long as its graph lives: the buffer must never be freed, even
            # when a larger shape replaces it later (see below). Zero-filled buffers stay valid for the graph because the
            # kernels return their counters to zero after every launch.
            _state.graph_held.add((device, key))
        return buf
    if capturing:
        # No buffer of this size exists yet and allocating a long-lived one inside a capture would tie it to the graph's
        # private pool: give this launch scratch of its own from that pool, which lives exactly as long as the graph
        # (a zero-filled one becomes a memset node on every replay). A step that ran eagerly once before it was captured
        # never gets here.
        alloc = max(int(nbytes), 256)
        return torch.zeros(alloc, dtype=torch.uint8, device=device) if zero else torch.empty(alloc, dtype=torch.uint8, device=device)
    if buf is not None and (device, key) in _state.graph_held:
        _state.retired.append(buf)          # a captured graph may still launch into it
        _state.graph_held.discard((device, key))
    alloc = max(int(nbytes), 256)
    with torch.inference_mode(False):   # kept across calls and cleared in place after a time-out
        buf = torch.zeros(alloc, dtype=torch.uint8, device=device) if zero else torch.empty(alloc, dtype=torch.uint8, device=device)
    _state.workspaces[(device, key)] = buf
    return buf


# ---------------------------------------------------------------------------------------------------
# (5) KV page writes
# ---------------------------------------------------------------------------------------------------
def store_kvcache_unified_layout(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                                 slot_mapping: torch.Tensor, model_type: str = "causal_lm", context=None) -> None:
    """Scatter new K/V rows into the unified pool `[pages, page_size, Hkv, D]` at `slot_mapping`; slot < 0 skips.

    Same contract as store_kvcache_unified_layout (.../ops/kv_cache_kernels.py:150-172), including its asserts.
    """
    device = _require_cuda(key, value, k_cache, v_cache, slot_mapping)
    n, num_heads, head_dim = key.shape
    d_total = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == d_total and v_cache.stride(1) == d_total
    assert n == slot_mapping.numel(), f"`N`: {n}, `slot_mapping.numel()`: {slot_mapping.numel()}"
    if slot_mapping.dtype != torch.int32:
        raise ValueError("slot_mapping must be int32")
    if key.dtype != k_cache.dtype or value.dtype != v_cache.dtype:
        raise ValueError("key/value dtype must match the cache dtype")
    num_slots = k_cache.shape[0] * k_cache.shape[1]
    check(_lib.load().pdllm_store_kvcache_unified(
        key.data_ptr(), value.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr(),
        n, d_total, key.stride(0), value.stride(0), key.element_size(), num_slots,
        status_word(device).data_ptr(), _stream(device)))


def store_kvcache_distinct_layout(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                                  slot_mapping: torch.Tensor, model_type: str = "causal_lm", context=None) -> None:
    """Scatter into the vLLM-style pool: K `[pages, Hkv, D/x, page_size, x]`, V `[pages, Hkv, D, page_size]`.

    Same contract as store_kvcache_distinct_layout (.../ops/kv_cache_kernels.py:109-147). With
    model_type='causal_lm' the reference treats the caches as unified-shaped; so does this.
    """
    if model_type == "causal_lm":
        return store_kvcache_unified_layout(key, value, k_cache, v_cache, slot_mapping, model_type, context)
    device = _require_cuda(key, value, k_cache, v_cache, slot_mapping)
    n_blks, n_heads, hdim_x, blk_sz, x = k_cache.shape
    hdim = hdim_x * x
    n = key.shape[0]
    assert hdim == key.shape[-1] and n_heads == key.shape[1]
    assert n == slot_mapping.numel()
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("distinct-layout caches must be contiguous")
    if slot_mapping.dtype != torch.int32:
        raise ValueError("slot_mapping must be int32")
    check(_lib.load().pdllm_store_kvcache_distinct(
        key.data_ptr(), value.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr(),
        n, n_heads, hdim, blk_sz, x, key.stride(0), value.stride(0), key.element_size(), n_blks,
        status_word(device).data_ptr(), _stream(device)))


def load_kvcache(k_cache: torch.Tensor, v_cache: torch.Tensor, context, k_new: torch.Tensor,
                 v_new: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Gather every cached page of every sequence plus the new rows into contiguous `[sum(ctx+new), Hkv, D]`.

    Same contract as load_kvcache (.../ops/kv_cache_kernels.py:278-327). The fused attention kernel does not
    need this gather; it exists because callers of the reference op table may still ask for it.
    `context` needs: block_tables, context_lens, seq_lens_ts, cu_seqlens_q, cu_seqlens_k.
    """
    device = _require_cuda(k_cache, v_cache, k_new, v_new)
    assert k_cache.shape == v_cache.shape
    assert k_new.shape == v_new.shape
    _, page_size, h_kv, head_dim = k_cache.shape
    num_seqs, max_pages = context.block_tables.shape
    cu_q, cu_k = context.cu_seqlens_q, context.cu_seqlens_k
    assert cu_q.shape == cu_k.shape
    assert cu_q.shape[0] == num_seqs + 1
    total_k = int(cu_k[-1].item())
    k_out = torch.empty((total_k, h_kv, head_dim), device=device, dtype=k_cache.dtype)
    v_out = torch.empty_like(k_out)
    if not (k_new.is_contiguous() and v_new.is_contiguous()):
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
    check(_lib.load().pdllm_load_kvcache(
        k_cache.data_ptr(), v_cache.data_ptr(), k_new.data_ptr(), v_new.data_ptr(),
        context.block_tables.data_ptr(), context.block_tables.stride(0), max_pages,
        cu_q.data_ptr(), cu_k.data_ptr(), context.context_lens.data_ptr(), num_seqs, h_kv, head_dim, page_size,
        k_cache.shape[0], k_new.stride(0), k_cache.element_size(), k_out.data_ptr(), v_out.data_ptr(), total_k,
        status_word(device).data_ptr(), _stream(device)))
    return k_out, v_out


# ---------------------------------------------------------------------------------------------------
# (3)+(1) attention
# ---------------------------------------------------------------------------------------------------
_IMPL_CODE = {"auto": _lib.ATTN_AUTO, "simt": _lib.ATTN_SIMT, "tc": _lib.ATTN_TC}
LAST_ATTENTION_USED_CLUSTERS = False   # whether the latest "tc" call took the few-rows form (clusters merge the KV splits)


def paged_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, output: torch.Tensor, *,
                    cu_seqlens_q: torch.Tensor, max_query_len: int,
                    key_cache: Optional[torch.Tensor] = None, value_cache: Optional[torch.Tensor] = None,
                    block_table: Optional[torch.Tensor] = None, seq_lens: Optional[torch.Tensor] = None,
                    max_seq_len: int = 0, sm_scale: Optional[float] = None, mask: Optional[torch.Tensor] = None,
                    causal: bool = False, bidirectional: bool = True, diffusion_blk_sz: int = 32,
                    impl: str = "auto", num_splits: int = 0, trace: Optional[torch.Tensor] = None) -> str:
    """New rows attend `[selected prefix pages (block-table order) ‖ new rows]`; writes `output` in place.

    query/output `[T, Hq, D]`, key/value `[T, Hkv, D]` (the new rows of all sequences, packed by
    `cu_seqlens_q`). Cache: unified `[pages, page_size, Hkv, D]` or distinct (K 5-D, V 4-D); None = no context.
    `seq_lens[s]` = context + new length. `mask` (bool `[q, q]`, sequence-local) and `bidirectional` follow
    the reference d2f kernel (.../ops/prefix_prefill.py:169-204); `causal=True` is the scoring mask
    (prefilling_dllm_eval/fastdllm_parallelcomp.py:950-961). Returns the kernel used: "tc" or "simt".
    """
    device = _require_cuda(query, key, value, output)
    if query.dim() != 3 or key.dim() != 3 or value.dim() != 3:
        raise ValueError(f"expected q/k/v as [tokens, heads, dim], got {tuple(query.shape)} / {tuple(key.shape)}")
    total_q, hq, d = query.shape
    hkv = key.shape[1]
    if key.shape[0] != total_q or value.shape != key.shape or output.shape != query.shape:
        raise ValueError("q/k/v/output shapes disagree")
    for name, t in (("query", query), ("key", key), ("value", value), ("output", output)):
        if t.stride(-1) != 1 or t.stride(1) != d:
            raise ValueError(f"{name} must have contiguous heads and head_dim")
        if t.dtype != query.dtype:
            raise ValueError("q/k/v/output must share one dtype")
    if cu_seqlens_q.dtype != torch.int32:
        raise ValueError("cu_seqlens_q must be int32")
    p = AttnParams()
    p.q, p.k_new, p.v_new, p.out = query.data_ptr(), key.data_ptr(), value.data_ptr(), output.data_ptr()
    p.q_stride, p.k_stride, p.v_stride, p.out_stride = query.stride(0), key.stride(0), value.stride(0), output.stride(0)
    p.cu_seqlens_q = cu_seqlens_q.data_ptr()
    p.num_seqs = cu_seqlens_q.numel() - 1
    p.total_q = total_q
    p.num_q_heads, p.num_kv_heads, p.head_dim = hq, hkv, d
    p.dtype = dtype_code(query.dtype)
    p.kv_layout = _lib.KV_NONE
    if key_cache is not None and key_cache.numel() > 0:
        _require_cuda(key_cache, value_cache, block_table, seq_lens)
        if block_table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
            raise ValueError("block_table and seq_lens must be int32")
        if key_cache.dtype != query.dtype or value_cache.dtype != query.dtype:
            raise NotImplementedError("KV cache dtype must equal the query dtype (fp8 caches are not built)")
        if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
            raise ValueError("KV caches must be contiguous")
        if key_cache.dim() == 5:
            p.kv_layout = _lib.KV_DISTINCT
            p.num_pages, _, _, p.page_size, p.x = key_cache.shape
        elif key_cache.dim() == 4:
            p.kv_layout = _lib.KV_UNIFIED
            p.num_pages, p.page_size = key_cache.shape[0], key_cache.shape[1]
            p.x = 1
        else:
            raise ValueError(f"unrecognised KV cache shape {tuple(key_cache.shape)}")
        p.k_cache, p.v_cache = key_cache.data_ptr(), value_cache.data_ptr()
        p.block_table = block_table.data_ptr()
        p.block_table_stride = block_table.stride(0)
        p.max_pages = block_table.shape[1]
        p.seq_lens = seq_lens.data_ptr()
    if mask is not None:
        _require_cuda(mask)
        if mask.dtype != torch.bool or mask.dim() != 2:
            raise ValueError("mask must be a 2-D bool tensor")
        p.mask = mask.data_ptr()
        p.mask_stride_m, p.mask_stride_n = mask.stride(0), mask.stride(1)
    p.mask_mode = _lib.MASK_CAUSAL if causal else _lib.MASK_BLOCK
    p.bidirectional = 1 if bidirectional else 0
    p.diffusion_blk = int(diffusion_blk_sz)
    p.max_query_len = int(max_query_len)
    p.max_seq_len = int(max_seq_len) if max_seq_len else int(max_query_len)
    p.sm_scale = float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(d)
    p.impl = _IMPL_CODE[impl]
    p.num_splits = int(num_splits)
    p.status = status_word(device).data_ptr()
    if trace is not None:  # profiling aid: zeroed int64 [8, 64, 16] buffer for the tcgen05 kernel's timestamps
        if trace.dtype != torch.int64 or trace.numel() < 8 * 64 * 16 or not trace.is_cuda:
            raise ValueError("trace must be a CUDA int64 tensor with at least 8*64*16 elements")
        p.trace = trace.data_ptr()
    lib = _lib.load()
    chosen = lib.pdllm_attn_select_impl(ctypes.byref(p))
    if chosen < 0:
        check(chosen)
    need = lib.pdllm_attn_workspace_bytes(ctypes.byref(p))
    if need < 0:
        check(int(need))
    if need > 0:
        # zero-filled when it is created; the kernel keeps its arrival counters at zero between launches
        ws = _workspace(device, "attn", int(need), zero=True)
        p.workspace, p.workspace_bytes, p.workspace_zeroed = ws.data_ptr(), ws.numel(), 1
    global LAST_ATTENTION_USED_CLUSTERS
    LAST_ATTENTION_USED_CLUSTERS = chosen == _lib.ATTN_TC and lib.pdllm_attn_uses_cluster_kernel(ctypes.byref(p)) == 1
    check(lib.pdllm_paged_attention(ctypes.byref(p), _stream(device)))
    return "tc" if chosen == _lib.ATTN_TC else "simt"


def diffusion_lm_parallel_flash_decoding(query, key, value, output, kv_cache_dtype, key_cache, value_cache, block_table,
                                         query_start_loc, seq_lens, max_seq_len, max_query_len, k_scale, v_scale,
                                         diffusion_blk_sz=32, alibi_slopes=None, sliding_window=None, sm_scale=None,
                                         mask=None, bidirectional=False) -> None:
    """Drop-in for chunked_prefill_paged_decode (.../ops/chunked_prefill_decoding_unified_kernel.py:220-274).

    Writes `output` in place. Besides the reference's distinct cache layout this also takes the unified
    `[pages, page_size, Hkv, D]` pool directly, which is what removes the per-layer load_kvcache gather.
    Not built: fp8 caches (k_scale/v_scale other than 1), ALiBi, sliding windows, and the causal-LM
    single-query branch (max_query_len == 1 of a causal model) — they raise NotImplementedError.
    """
    if sm_scale is None:
        sm_scale = 1.0 / (query.shape[1] ** 0.5)  # sic: the reference divides by sqrt(num_heads) here
    if alibi_slopes is not None:
        raise NotImplementedError("alibi_slopes is not supported")
    if sliding_window is not None and sliding_window > 0:
        raise NotImplementedError("sliding_window is not supported")
    if "fp8" in str(kv_cache_dtype):
        raise NotImplementedError("fp8 KV caches are not supported")
    for scale in (k_scale, v_scale):
        if isinstance(scale, torch.Tensor):
            continue  # only read by the reference for fp8 caches
        if scale is not None and float(scale) != 1.0:
            raise NotImplementedError("k_scale / v_scale other than 1.0 are not supported")
    if mask is not None and isinstance(mask, (list, tuple)):
        raise ValueError("mask must be a tensor")
    seq_lens_t = seq_lens
    if not isinstance(seq_lens_t, torch.Tensor):
        seq_lens_t = torch.tensor(list(seq_lens), dtype=torch.int32, device=query.device)
    paged_attention(query, key, value, output, cu_seqlens_q=query_start_loc, max_query_len=int(max_query_len),
                    key_cache=key_cache, value_cache=value_cache, block_table=block_table,
                    seq_lens=seq_lens_t.to(torch.int32), max_seq_len=int(max_seq_len) if max_seq_len else 0,
                    sm_scale=sm_scale, mask=mask, causal=False, bidirectional=bool(bidirectional),
                    diffusion_blk_sz=int(diffusion_blk_sz))


# ---------------------------------------------------------------------------------------------------
# (4) unmask step
# ---------------------------------------------------------------------------------------------------
def unmask_step(logits: torch.Tensor, block_ids: torch.Tensor, *, mask_token_id: int, threshold: float,
                last_logit: Optional[torch.Tensor] = None, shift: bool = True,
                softmax_dtype: Optional[torch.dtype] = None, return_details: bool = False):
    """One confidence-threshold denoise step on `block_ids` (int64 `[block_len]`, updated in place).

    Fuses _shift_logits + sample_tokens (greedy) + the top-1/threshold transfer loop of
    prefilling_dllm_eval/fastdllm_parallelcomp.py:1007-1015, 204-233, 2422-2440 and
    prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py:1648-1681, 2143-2157.
    `softmax_dtype=torch.float32` reproduces the engine (fp32 softmax); `None` uses the logits dtype like the
    eval path, including its rounding of the probability and of the threshold before `>=`.
    Returns a device int32 tensor `[candidates_before, filled, candidates_left]` (no host sync), plus
    per-slot confidence and arg-max when `return_details`.
    """
    device = _require_cuda(logits, block_ids)
    if logits.dim() != 2:
        raise ValueError(f"logits must be [block_len, vocab], got {tuple(logits.shape)}")
    block_len, vocab = logits.shape
    if block_ids.dtype != torch.int64 or block_ids.numel() != block_len or not block_ids.is_contiguous():
        raise ValueError("block_ids must be a contiguous int64 tensor with one entry per logits row")
    if logits.stride(1) != 1:
        raise ValueError("logits rows must be contiguous")
    if last_logit is not None:
        last_logit = last_logit.reshape(-1)
        if last_logit.numel() != vocab or last_logit.dtype != logits.dtype or not last_logit.is_contiguous():
            raise ValueError("last_logit must be a contiguous [vocab] tensor of the logits dtype")
    conf_dtype = dtype_code(softmax_dtype if softmax_dtype is not None else logits.dtype)
    lib = _lib.load()
    ws_bytes = int(lib.pdllm_unmask_workspace_bytes(block_len))
    ws = _workspace(device, f"unmask{block_len}", ws_bytes, zero=True)
    counts = torch.empty(3, dtype=torch.int32, device=device)
    conf = torch.empty(block_len, dtype=torch.float32, device=device) if return_details else None
    x0 = torch.empty(block_len, dtype=torch.int64, device=device) if return_details else None
    check(lib.pdllm_unmask_step(logits.data_ptr(), logits.stride(0), _ptr(last_logit), dtype_code(logits.dtype), block_len,
                                vocab, 1 if shift else 0, block_ids.data_ptr(), int(mask_token_id), float(threshold),
                                conf_dtype, counts.data_ptr(), _ptr(conf), _ptr(x0), ws.data_ptr(), ws.numel(),
                                _stream(device)))
    if return_details:
        return counts, conf, x0
    return counts


def unmask_step_batched(logits: torch.Tensor, block_ids: torch.Tensor, *, mask_token_id: int, threshold: float,
                        last_logit: Optional[torch.Tensor] = None, shift: bool = True,
                        softmax_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """`unmask_step` for several requests that share a denoise step, in one launch.

    logits `[batch, block_len, vocab]` (any batch stride, contiguous rows), block_ids int64 `[batch, block_len]` contiguous
    (updated in place), last_logit `[batch, vocab]` or None. Returns int32 `[batch, 3]` counts on the device.
    """
    device = _require_cuda(logits, block_ids)
    if logits.dim() != 3 or logits.stride(2) != 1:
        raise ValueError(f"logits must be [batch, block_len, vocab] with contiguous rows, got {tuple(logits.shape)}")
    batch, block_len, vocab = logits.shape
    if block_ids.dtype != torch.int64 or tuple(block_ids.shape) != (batch, block_len) or not block_ids.is_contiguous():
        raise ValueError("block_ids must be a contiguous int64 [batch, block_len] tensor")
    last_stride = 0
    if last_logit is not None:
        if tuple(last_logit.shape) != (batch, vocab) or last_logit.dtype != logits.dtype or last_logit.stride(1) != 1:
            raise ValueError("last_logit must be [batch, vocab] of the logits dtype with contiguous rows")
        last_stride = last_logit.stride(0)
    conf_dtype = dtype_code(softmax_dtype if softmax_dtype is not None else logits.dtype)
    lib = _lib.load()
    ws_bytes = batch * int(lib.pdllm_unmask_workspace_bytes(block_len))
    ws = _workspace(device, f"unmask{block_len}x{batch}", ws_bytes, zero=True)
    counts = torch.empty((batch, 3), dtype=torch.int32, device=device)
    check(lib.pdllm_unmask_step_batched(logits.data_ptr(), logits.stride(1), logits.stride(0), _ptr(last_logit), last_stride,
                                        dtype_code(logits.dtype), batch, block_len, vocab, 1 if shift else 0, block_ids.data_ptr(),
                                        int(mask_token_id), float(threshold), conf_dtype, counts.data_ptr(), None, None,
                                        ws.data_ptr(), ws.numel(), _stream(device)))
    return counts


# ---------------------------------------------------------------------------------------------------
# (2) scoring, selection, eviction
# ---------------------------------------------------------------------------------------------------
def self_information_scores(label_rows: torch.Tensor, labels: torch.Tensor, n_chunks: int,
                            return_nll: bool = False):
    """score[c] = mean_i log_softmax(label_rows[c, i])[labels[i]] in fp32 (non-finite → -inf).

    label_rows: `[n_chunks * n_labels, vocab]` logits already gathered at `label_position - 1`.
    The tail of score_chunks_self_information_batched (prefilling_dllm_eval/fastdllm_parallelcomp.py:1415-1422).
    """
    device = _require_cuda(label_rows, labels)
    if label_rows.dim() != 2 or label_rows.stride(1) != 1:
        raise ValueError("label_rows must be [rows, vocab] with contiguous rows")
    n_labels = labels.numel()
    if labels.dtype != torch.int64 or not labels.is_contiguous():
        raise ValueError("labels must be contiguous int64")
    if label_rows.shape[0] != n_chunks * n_labels:
        raise ValueError(f"expected {n_chunks * n_labels} rows, got {label_rows.shape[0]}")
    scores = torch.empty(n_chunks, dtype=torch.float32, device=device)
    nll = torch.empty(max(1, n_chunks * n_labels), dtype=torch.float32, device=device)
    check(_lib.load().pdllm_self_information_scores(
        label_rows.data_ptr(), label_rows.stride(0), dtype_code(label_rows.dtype), n_chunks, n_labels, label_rows.shape[1],
        labels.data_ptr(), scores.data_ptr(), nll.data_ptr(), status_word(device).data_ptr(), _stream(device)))
    if return_nll:
        return scores, nll[: n_chunks * n_labels].view(n_chunks, n_labels)
    return scores


def topk_chunks(scores: torch.Tensor, topk: int, keep_first_chunk: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """Stable top-K (ties keep the lower index), returned ascending: (selected int32 `[n]`, count int32 `[1]`).

    The ranking of select_chunks (prefilling_dllm_eval/fastdllm_parallelcomp.py:1949-1953).
    """
    device = _require_cuda(scores)
    if scores.dtype != torch.float32 or scores.dim() != 1 or not scores.is_contiguous():
        raise ValueError("scores must be a contiguous fp32 vector")
    n = scores.numel()
    selected = torch.empty(max(1, n), dtype=torch.int32, device=device)
    count = torch.zeros(1, dtype=torch.int32, device=device)
    check(_lib.load().pdllm_topk_chunks(scores.data_ptr(), n, int(topk), 1 if keep_first_chunk else 0, selected.data_ptr(),
                                        count.data_ptr(), _stream(device)))
    return selected, count


def query_to_chunk_attention_scores(q: torch.Tensor, k: torch.Tensor, *, prefix_len: int, chunk_len: int,
                                    query_len: int, scale: float, reduce_mode: str = "sum",
                                    attention_mask: str = "causal", block_n: int = 64,
                                    block_chunk: int = 64) -> torch.Tensor:
    """Per-query-head query→chunk attention mass, fp32 `[Hq, chunk_len]`.

    Drop-in for query_to_chunk_attention_scores (.../ops/triton_eviction_scorer.py:114-210): same checks, same
    exception types. `block_n` / `block_chunk` are accepted for signature parity and ignored.
    """
    if not q.is_cuda or not k.is_cuda:
        raise ValueError("Triton eviction scorer requires CUDA tensors.")
    if q.ndim != 3 or k.ndim != 3:
        raise ValueError(f"Expected q/k as [seq, heads, dim], got {tuple(q.shape)} / {tuple(k.shape)}")
    if chunk_len <= 0 or query_len <= 0:
        return torch.empty(0, device=q.device)
    if int(q.shape[0]) != int(k.shape[0]):
        raise ValueError("q and k must use the same sequence length.")
    num_query_heads, num_kv_heads, head_dim = int(q.shape[1]), int(k.shape[1]), int(q.shape[2])
    if int(k.shape[2]) != head_dim:
        raise ValueError("q and k must use the same head dimension.")
    if num_query_heads % num_kv_heads != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads.")
    if head_dim > 256:
        raise ValueError(f"Unsupported head_dim for Triton eviction scorer: {head_dim}")
    if query_len > 64:
        raise ValueError(f"query_len={query_len} is too large for first Triton scorer version.")
    mask = (attention_mask or "full").lower()
    if mask in {"full", "none", "query_to_chunk"}:
        causal = 0
    elif mask == "causal":
        causal = 1
    else:
        raise ValueError(f"Unsupported token attention mask for Triton scorer: {attention_mask}")
    if q.dtype != k.dtype:
        raise ValueError("q and k must share one dtype")
    q, k = q.contiguous(), k.contiguous()
    device = q.device
    key_len = int(k.shape[0])
    out = torch.empty((num_query_heads, int(chunk_len)), device=device, dtype=torch.float32)
    lib = _lib.load()
    ws_bytes = int(lib.pdllm_evict_workspace_bytes(num_query_heads, int(query_len), key_len))
    ws = _workspace(device, "evict", ws_bytes)
    check(lib.pdllm_query_to_chunk_scores(q.data_ptr(), k.data_ptr(), dtype_code(q.dtype), key_len, num_query_heads,
                                          num_kv_heads, head_dim, int(prefix_len), int(chunk_len), int(query_len),
                                          float(scale), 1 if (reduce_mode or "sum").lower() == "mean" else 0, causal,
                                          out.data_ptr(), ws.data_ptr(), ws.numel(), _stream(device)))
    return out


def evict_select(head_scores: torch.Tensor, *, num_kv_heads: int, keep_count: int, pool_kernel: int = 7,
                 per_head: bool = False, force_keep_first: bool = True, keep_high: bool = True,
                 return_pooled: bool = False):
    """Pool, reduce and rank `[n_layers, Hq, chunk_len]` head scores into ascending kept positions (int64).

    global  → `[1, keep_count]`: maxpool → sum over heads → mean over layers → BOS + top-(keep_count-1)
              (prefilling_dllm_eval/fastdllm_parallelcomp.py:1607-1637, 1997-2023);
    per_head → `[n_layers, Hkv, keep_count]`: maxpool → mean over each KV group (:1742-1760, engine
              fastdllm_engine.py:1396-1432, 904-927).
    """
    device = _require_cuda(head_scores)
    if head_scores.dtype != torch.float32 or head_scores.dim() != 3 or not head_scores.is_contiguous():
        raise ValueError("head_scores must be contiguous fp32 [n_layers, Hq, chunk_len]")
    n_layers, hq, chunk_len = head_scores.shape
    rows = n_layers * num_kv_heads if per_head else 1
    keep = torch.empty((rows, keep_count), dtype=torch.int64, device=device)
    pooled = torch.empty((rows, chunk_len), dtype=torch.float32, device=device) if return_pooled else None
    check(_lib.load().pdllm_evict_select(head_scores.data_ptr(), n_layers, hq, int(num_kv_heads), chunk_len, int(pool_kernel),
                                         1 if per_head else 0, int(keep_count), 1 if force_keep_first else 0,
                                         1 if keep_high else 0, keep.data_ptr(), _ptr(pooled), _stream(device)))
    if per_head:
        keep = keep.view(n_layers, num_kv_heads, keep_count)
        if pooled is not None:
            pooled = pooled.view(n_layers, num_kv_heads, chunk_len)
    if return_pooled:
        return keep, pooled
    return keep


# ---------------------------------------------------------------------------------------------------
# prefill/decode boundary: page <-> dense copies
# ---------------------------------------------------------------------------------------------------
def _page_ids_tensor(page_ids, device: torch.device) -> torch.Tensor:
    if isinstance(page_ids, torch.Tensor):
        return page_ids.to(device=device, dtype=torch.int32).contiguous()
    return torch.tensor(list(page_ids), dtype=torch.int32, device=device)


def gather_pages(cache: torch.Tensor, page_ids, n_tokens: int) -> torch.Tensor:
    """Dense `[n_tokens, Hkv, D]` copy of the first n_tokens held by `page_ids` of a unified pool."""
    device = _require_cuda(cache)
    _, page_size, hkv, d = cache.shape
    out = torch.empty((n_tokens, hkv, d), dtype=cache.dtype, device=device)
    ids = _page_ids_tensor(page_ids, device)
    if n_tokens > ids.numel() * page_size:
        raise ValueError("n_tokens exceeds the capacity of page_ids")
    check(_lib.load().pdllm_gather_pages(cache.data_ptr(), ids.data_ptr(), n_tokens, page_size, hkv * d, cache.element_size(),
                                         cache.shape[0], out.data_ptr(), status_word(device).data_ptr(), _stream(device)))
    return out


def scatter_pages(src: torch.Tensor, cache: torch.Tensor, page_ids) -> None:
    """Write dense `[n_tokens, Hkv, D]` rows into the pages `page_ids` of a unified pool."""
    device = _require_cuda(cache, src)
    _, page_size, hkv, d = cache.shape
    n_tokens = src.shape[0]
    if tuple(src.shape[1:]) != (hkv, d) or src.dtype != cache.dtype:
        raise ValueError(f"source rows {tuple(src.shape)} do not match the pool rows ({hkv}, {d})")
    src = src.contiguous()
    ids = _page_ids_tensor(page_ids, device)
    if n_tokens > ids.numel() * page_size:
        raise ValueError("n_tokens exceeds the capacity of page_ids")
    check(_lib.load().pdllm_scatter_pages(src.data_ptr(), ids.data_ptr(), n_tokens, page_size, hkv * d, cache.element_size(),
                                          cache.shape[0], cache.data_ptr(), status_word(device).data_ptr(), _stream(device)))


def compact_pages_per_head(cache: torch.Tensor, src_page_ids, dst_page_ids, keep: torch.Tensor, *, src_tokens: int,
                           dst_start: int = 0) -> None:
    """Per-KV-head compaction: dst token `dst_start + j` of head h := src token `keep[h, j]` (in place is fine)."""
    device = _require_cuda(cache, keep)
    _, page_size, hkv, d = cache.shape
    if keep.dim() != 2 or keep.shape[0] != hkv:
        raise ValueError(f"keep must be [num_kv_heads={hkv}, keep_count], got {tuple(keep.shape)}")
    keep = keep.to(torch.int64).contiguous()
    keep_count = keep.shape[1]
    src_ids = _page_ids_tensor(src_page_ids, device)
    dst_ids = _page_ids_tensor(dst_page_ids, device)
    staging = _workspace(device, "compact", keep_count * hkv * d * cache.element_size())
    check(_lib.load().pdllm_compact_pages_per_head(cache.data_ptr(), src_ids.data_ptr(), dst_ids.data_ptr(), keep.data_ptr(),
                                                   keep_count, int(src_tokens), int(dst_start), dst_ids.numel() * page_size, page_size, hkv, d,
                                                   cache.element_size(), cache.shape[0], staging.data_ptr(),
                                                   status_word(device).data_ptr(), _stream(device)))


def rope_pages(k_cache: torch.Tensor, page_ids, start: int, cos: torch.Tensor, sin: torch.Tensor) -> None:
    """Rotate, in place, the K rows of tokens `[start, start + n)` of a unified pool that were stored un-rotated.

    cos / sin: `[n, D]` (or `[n, 1, D]`) tables in the cache dtype. Used after a per-head compaction, where kept row j of
    every head takes position j of the compacted span (reference eval class :2284-2288, :2890-2912)."""
    device = _require_cuda(k_cache, cos, sin)
    _, page_size, hkv, d = k_cache.shape
    cos = cos.reshape(-1, d).contiguous()
    sin = sin.reshape(-1, d).contiguous()
    n = cos.shape[0]
    if sin.shape != cos.shape or cos.dtype != k_cache.dtype or sin.dtype != k_cache.dtype:
        raise ValueError("cos / sin must be [n, head_dim] tables in the cache dtype")
    ids = _page_ids_tensor(page_ids, device)
    if start < 0 or start + n > ids.numel() * page_size:
        raise ValueError("token range exceeds the capacity of page_ids")
    check(_lib.load().pdllm_rope_pages(k_cache.data_ptr(), ids.data_ptr(), int(start), n, cos.data_ptr(), sin.data_ptr(), page_size,
                                       hkv, d, dtype_code(k_cache.dtype), k_cache.shape[0], status_word(device).data_ptr(),
                                       _stream(device)))


# ---------------------------------------------------------------------------------------------------
# row-wise pieces of the transformer block
# ---------------------------------------------------------------------------------------------------
def add_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, delta: Optional[torch.Tensor] = None) -> torch.Tensor:
    """`x += delta` in place when `delta` is given, then returns RMSNorm(x) * weight (new tensor). x, delta: `[T, hidden]`."""
    device = _require_cuda(x, weight, delta)
    if x.dim() != 2 or x.stride(1) != 1 or weight.numel() != x.shape[1] or not weight.is_contiguous():
        raise ValueError("add_rmsnorm expects x [tokens, hidden] with contiguous rows and weight [hidden]")
    if delta is not None and (delta.shape != x.shape or delta.stride(1) != 1 or delta.dtype != x.dtype):
        raise ValueError("delta must match x")
    out = torch.empty((x.shape[0], x.shape[1]), dtype=x.dtype, device=device)
    check(_lib.load().pdllm_add_rmsnorm(x.data_ptr(), _ptr(delta), weight.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1], x.stride(0),
                                        0 if delta is None else delta.stride(0), out.stride(0), float(eps), dtype_code(x.dtype),
                                        _stream(device)))
    return out


def rope_inplace(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> None:
    """Rotate the heads of `x` `[T, heads, D]` (any row stride; heads and D contiguous) in place with tables `[T, D]`."""
    device = _require_cuda(x, cos, sin)
    t, h, d = x.shape
    if x.stride(2) != 1 or x.stride(1) != d:
        raise ValueError("x must have contiguous heads and head_dim")
    cos, sin = cos.reshape(-1, d), sin.reshape(-1, d)
    if cos.shape[0] != t or sin.shape != cos.shape or cos.dtype != x.dtype or sin.dtype != x.dtype or not (cos.is_contiguous() and sin.is_contiguous()):
        raise ValueError("cos / sin must be contiguous [tokens, head_dim] tables in the dtype of x")
    check(_lib.load().pdllm_rope_inplace(x.data_ptr(), cos.data_ptr(), sin.data_ptr(), t, h, d, x.stride(0), dtype_code(x.dtype), _stream(device)))


def rope_store(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, num_q_heads: int, num_kv_heads: int,
               k_cache: Optional[torch.Tensor] = None, v_cache: Optional[torch.Tensor] = None, slot_mapping: Optional[torch.Tensor] = None,
               *, k_before_rotation: bool = False) -> None:
    """Rotate the q and k heads of `qkv` `[T, Hq + 2 Hkv, D]` (any row stride) in place and, when `slot_mapping` is given, write
    its k and v heads into the unified pools `k_cache` / `v_cache` `[pages, page_size, Hkv, D]` — the model's rotary embedding and
    `store_kvcache_unified_layout` (.../models/dream.py:75-76, .../layers/attention/attention_v4.py:330-331) in one launch.
    bf16 / fp16 with D a multiple of 16; other inputs raise NotImplementedError (use `rope_inplace` + the store op)."""
    device = _require_cuda(qkv, cos, sin, k_cache, v_cache, slot_mapping)
    t, heads, d = qkv.shape
    if heads != num_q_heads + 2 * num_kv_heads or qkv.stride(2) != 1 or qkv.stride(1) != d:
        raise ValueError("qkv must be [T, Hq + 2 Hkv, D] with contiguous heads and head_dim")
    cos, sin = cos.reshape(-1, d), sin.reshape(-1, d)
    if cos.shape[0] != t or sin.shape != cos.shape or cos.dtype != qkv.dtype or sin.dtype != qkv.dtype or not (cos.is_contiguous() and sin.is_contiguous()):
        raise ValueError("cos / sin must be contiguous [tokens, head_dim] tables in the dtype of qkv")
    num_slots = 0
    if slot_mapping is not None:
        if k_cache is None or v_cache is None or k_cache.shape != v_cache.shape or k_cache.dim() != 4:
            raise ValueError("the page write needs k_cache and v_cache [pages, page_size, Hkv, D]")
        if tuple(k_cache.shape[2:]) != (num_kv_heads, d) or k_cache.dtype != qkv.dtype or not (k_cache.is_contiguous() and v_cache.is_contiguous()):
            raise ValueError("caches must be contiguous [pages, page_size, Hkv, D] pools of the dtype of qkv")
        if slot_mapping.dtype != torch.int32 or slot_mapping.numel() != t or not slot_mapping.is_contiguous():
            raise ValueError("slot_mapping must be a contiguous int32 [T] tensor")
        num_slots = k_cache.shape[0] * k_cache.shape[1]
    check(_lib.load().pdllm_rope_store(qkv.data_ptr(), qkv.stride(0), cos.data_ptr(), sin.data_ptr(), t, num_q_heads, num_kv_heads, d,
                                       _ptr(k_cache) if slot_mapping is not None else None, _ptr(v_cache) if slot_mapping is not None else None,
                                       _ptr(slot_mapping), num_slots, 1 if k_before_rotation else 0, dtype_code(qkv.dtype),
                                       status_word(device).data_ptr(), _stream(device)))


LINEAR_WEIGHTS_AT_REST = 0x100      # PDLLM_LINEAR_WEIGHTS_AT_REST


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, *, silu_mul_interleaved: bool = False,
           out: Optional[torch.Tensor] = None, weights_at_rest: bool = False) -> torch.Tensor:
    """`x @ weight.T (+ bias)` on the tcgen05 GEMM kernel: x `[M, K]`, weight `[N, K]` (the nn.Linear layout), bf16 / fp16.

    silu_mul_interleaved: `weight` holds gate and up rows interleaved (row 2i = gate_i, 2i + 1 = up_i) and the result is
    `silu(gate) * up`, `[M, N / 2]`, with the rounding of the unfused projection -> activation -> product sequence.
    weights_at_rest: nothing still in flight on the stream writes `weight` (model weights after loading): the kernel may start
    streaming them while the kernel before it on the stream is still finishing.
    Takes the place of F.linear in QKVParallelLinear / MergedColumnParallelLinear / RowParallelLinear / ParallelLMHead
    (prefilling_dllm_engine/prefilling_dllm/layers/linear.py:108-244, layers/embed_head.py:63-74)."""
    device = _require_cuda(x, weight, bias)
    if x.dim() != 2 or weight.dim() != 2 or x.shape[1] != weight.shape[1]:
        raise ValueError(f"linear expects x [M, K] and weight [N, K], got {tuple(x.shape)} and {tuple(weight.shape)}")
    if x.stride(1) != 1 or weight.stride(1) != 1 or x.dtype != weight.dtype:
        raise ValueError("x and weight must have contiguous rows and one dtype")
    m, k = x.shape
    n = weight.shape[0]
    if bias is not None and (bias.numel() != n or bias.dtype != x.dtype or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous [N] tensor of the dtype of x")
    cols = n // 2 if silu_mul_interleaved else n
    if out is None:
        out = torch.empty((m, cols), dtype=x.dtype, device=device)
    elif tuple(out.shape) != (m, cols) or out.stride(1) != 1 or out.dtype != x.dtype:
        raise ValueError("out must be [M, N] (or [M, N / 2] with the fused activation) with contiguous rows")
    if m == 0:
        return out
    lib = _lib.load()
    need = int(lib.pdllm_linear_workspace_bytes(m, n, k))
    ws_ptr, ws_bytes = None, 0
    if need > 0:
        ws = _workspace(device, "linear", need, zero=True)   # zero-filled at creation; the kernel keeps its counters at zero
        ws_ptr, ws_bytes = ws.data_ptr(), ws.numel()
    check(lib.pdllm_linear(x.data_ptr(), x.stride(0), weight.data_ptr(), weight.stride(0), _ptr(bias), out.data_ptr(), out.stride(0),
                           m, n, k, dtype_code(x.dtype), (1 if silu_mul_interleaved else 0) | (LINEAR_WEIGHTS_AT_REST if weights_at_rest else 0),
                           ws_ptr, ws_bytes, 1,
                           status_word(device).data_ptr(), _stream(device)))
    return out


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """`silu(gate_up[:, :I]) * gate_up[:, I:]` for `[T, 2I]` rows."""
    device = _require_cuda(gate_up)
    if gate_up.dim() != 2 or gate_up.stride(1) != 1 or gate_up.shape[1] % 2 != 0:
        raise ValueError("gate_up must be [tokens, 2 * intermediate] with contiguous rows")
    inter = gate_up.shape[1] // 2
    out = torch.empty((gate_up.shape[0], inter), dtype=gate_up.dtype, device=device)
    check(_lib.load().pdllm_silu_mul(gate_up.data_ptr(), out.data_ptr(), gate_up.shape[0], inter, gate_up.stride(0), out.stride(0),
                                     dtype_code(gate_up.dtype), _stream(device)))
    return out



def copy_pages(src_cache: torch.Tensor, src_page_ids: torch.Tensor, dst_cache: torch.Tensor, dst_page_ids: torch.Tensor, *,
               n_lists: int, tokens_per_list: int) -> None:
    """Pool to pool copy of `n_lists` page lists (`tokens_per_list` tokens each); `src_cache` may live on another GPU.

    Launched on the device of `dst_cache`; both id tensors (int32) must be on that device. When the pools are on
    different GPUs the source is read through peer access, straight across NVLink."""
    device = _require_cuda(dst_cache, src_page_ids, dst_page_ids)
    if not src_cache.is_cuda:
        raise ValueError("pdllm_b200 ops require CUDA tensors (there is no CPU path)")
    if src_cache.dim() != 4 or dst_cache.dim() != 4 or src_cache.shape[1:] != dst_cache.shape[1:] or src_cache.dtype != dst_cache.dtype:
        raise ValueError("pools must be unified [pages, page_size, Hkv, D] of one shape per page and one dtype")
    if src_page_ids.dtype != torch.int32 or dst_page_ids.dtype != torch.int32 or src_page_ids.numel() != dst_page_ids.numel():
        raise ValueError("page id lists must be int32 and of equal length")
    _, page_size, hkv, d = dst_cache.shape
    per_list = -(-int(tokens_per_list) // page_size)
    if src_page_ids.numel() != int(n_lists) * per_list:
        raise ValueError(f"expected {int(n_lists) * per_list} page ids, got {src_page_ids.numel()}")
    lib = _lib.load()
    if src_cache.device != device:
        check(lib.pdllm_enable_peer_access(device.index, src_cache.device.index))
    with torch.cuda.device(device):
        check(lib.pdllm_copy_pages(src_cache.data_ptr(), src_page_ids.contiguous().data_ptr(), dst_cache.data_ptr(),
                                   dst_page_ids.contiguous().data_ptr(), int(n_lists), int(tokens_per_list), page_size, hkv * d,
                                   dst_cache.element_size(), src_cache.shape[0], dst_cache.shape[0], status_word(device).data_ptr(),
                                   _stream(device)))
