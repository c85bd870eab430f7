"""Per-thread forward context for callers that drive the op table the way the reference attention layer does.

The reference keeps the metadata of the running forward (cu_seqlens, slot mapping, block tables, context lengths) in a
`threading.local` so that a prefill on the `pd-prefetch` thread and a decode on the main thread do not see each
other's state (prefilling_dllm_engine/prefilling_dllm/utils/context.py:27, :56-139). The kernels here take all of it as
arguments; this module only offers the same three calls for integrations that still pass a `context` object to
`ops.load_kvcache` / `ops.store_kvcache_*`.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Any, List, Optional

import torch

_THREAD = threading.local()


@dataclass
class ContextForDiffusionLM:
    is_prefill: bool = False
    cu_seqlens_q: Optional[torch.Tensor] = None
    cu_seqlens_k: Optional[torch.Tensor] = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: Optional[torch.Tensor] = None
    context_lens: Optional[torch.Tensor] = None
    block_tables: Optional[torch.Tensor] = None
    seqs: Optional[List[Any]] = None
    seq_lens: Optional[List[int]] = None
    seq_lens_ts: Optional[torch.Tensor] = None
    kv_cache_layout: str = "unified"
    need_kv_cache_store: bool = True
    block_mask: Any = None
    decode_delta_state: Any = None
    prefill_sparse_state: Any = None

    def __post_init__(self) -> None:
        self.total_lens = None
        if self.seq_lens_ts is not None and self.context_lens is not None:
            self.total_lens = self.seq_lens_ts + self.context_lens


def get_context_diffusion_lm() -> ContextForDiffusionLM:
    ctx = getattr(_THREAD, "diffusion_lm", None)
    if ctx is None:
        ctx = ContextForDiffusionLM()
        _THREAD.diffusion_lm = ctx
    return ctx


def set_context_diffusion_lm(is_prefill, **fields) -> None:
    _THREAD.diffusion_lm = ContextForDiffusionLM(is_prefill=bool(is_prefill), **fields)


def reset_context_diffusion_lm() -> None:
    _THREAD.diffusion_lm = ContextForDiffusionLM()
