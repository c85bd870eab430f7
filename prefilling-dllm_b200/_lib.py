"""ctypes binding of libpdllm_b200.so (the C-ABI declared in include/pdllm_b200.h).

The library is the product path: if it is missing or does not load, importing an op raises — there is no
CPU or PyTorch fallback behind these calls.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_int32, c_int64, c_void_p

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libpdllm_b200.so")

ABI_VERSION = 5
# dtype codes
F32, BF16, F16 = 0, 1, 2
# cache layouts
KV_NONE, KV_UNIFIED, KV_DISTINCT = 0, 1, 2
# mask modes
MASK_BLOCK, MASK_CAUSAL = 0, 1
# attention implementations
ATTN_AUTO, ATTN_SIMT, ATTN_TC = 0, 1, 2
# host error codes
E_INVALID, E_UNSUPPORTED, E_WORKSPACE, E_DRIVER = -1, -2, -3, -4
# device status codes
S_OK, S_BAD_SLOT, S_BAD_PAGE, S_BAD_LABEL, S_BAD_INDEX, S_WAIT_TIMEOUT = 0, 1, 2, 3, 4, 8

STATUS_NAMES = {
    S_OK: "ok",
    S_BAD_SLOT: "slot_mapping entry out of range",
    S_BAD_PAGE: "block_table entry out of range",
    S_BAD_LABEL: "label id out of range",
    S_BAD_INDEX: "keep index out of range",
    S_WAIT_TIMEOUT: "bounded device wait expired",
}


class AttnParams(Structure):
    """Mirror of `pdllm_attn_params`."""

    _fields_ = [
        ("q", c_void_p), ("k_new", c_void_p), ("v_new", c_void_p), ("out", c_void_p),
        ("k_cache", c_void_p), ("v_cache", c_void_p),
        ("block_table", c_void_p), ("cu_seqlens_q", c_void_p), ("seq_lens", c_void_p),
        ("mask", c_void_p), ("status", c_void_p), ("workspace", c_void_p), ("trace", c_void_p),
        ("workspace_bytes", c_int64),
        ("q_stride", c_int64), ("k_stride", c_int64), ("v_stride", c_int64), ("out_stride", c_int64),
        ("block_table_stride", c_int64),
        ("mask_stride_m", c_int64), ("mask_stride_n", c_int64),
        ("num_pages", c_int64), ("total_q", c_int64),
        ("num_seqs", c_int32), ("max_pages", c_int32),
        ("num_q_heads", c_int32), ("num_kv_heads", c_int32), ("head_dim", c_int32),
        ("page_size", c_int32), ("x", c_int32),
        ("kv_layout", c_int32), ("dtype", c_int32), ("mask_mode", c_int32),
        ("bidirectional", c_int32), ("diffusion_blk", c_int32),
        ("max_query_len", c_int32), ("max_seq_len", c_int32),
        ("impl", c_int32), ("num_splits", c_int32),
        ("sm_scale", c_float),
        ("workspace_zeroed", c_int32),
    ]


_SIGNATURES = {
    "pdllm_abi_version": (c_int, []),
    "pdllm_last_error": (c_char_p, []),
    "pdllm_device_supported": (c_int, []),
    "pdllm_store_kvcache_unified": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                            c_int64, c_int, c_int64, c_void_p, c_void_p]),
    "pdllm_store_kvcache_distinct": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int,
                                             c_int, c_int64, c_int64, c_int, c_int64, c_void_p, c_void_p]),
    "pdllm_load_kvcache": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p,
                                   c_void_p, c_int, c_int, c_int, c_int, c_int64, c_int64, c_int, c_void_p, c_void_p,
                                   c_int64, c_void_p, c_void_p]),
    "pdllm_attn_workspace_bytes": (c_int64, [POINTER(AttnParams)]),
    "pdllm_paged_attention": (c_int, [POINTER(AttnParams), c_void_p]),
    "pdllm_attn_select_impl": (c_int, [POINTER(AttnParams)]),
    "pdllm_attn_uses_cluster_kernel": (c_int, [POINTER(AttnParams)]),
    "pdllm_unmask_workspace_bytes": (c_int64, [c_int]),
    "pdllm_unmask_step": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_int64, c_int, c_void_p, c_int64, c_float,
                                  c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "pdllm_unmask_step_batched": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int, c_int, c_int, c_int64, c_int, c_void_p,
                                          c_int64, c_float, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "pdllm_unmask_step_static": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_int64, c_int, c_void_p, c_int64, c_float,
                                         c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "pdllm_self_information_scores": (c_int, [c_void_p, c_int64, c_int, c_int, c_int, c_int64, c_void_p, c_void_p,
                                              c_void_p, c_void_p, c_void_p]),
    "pdllm_topk_chunks": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "pdllm_evict_workspace_bytes": (c_int64, [c_int, c_int, c_int64]),
    "pdllm_query_to_chunk_scores": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_int, c_int, c_int, c_int,
                                            c_float, c_int, c_int, c_void_p, c_void_p, c_int64, c_void_p]),
    "pdllm_evict_select": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                   c_void_p, c_void_p]),
    "pdllm_gather_pages": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int64, c_int, c_int64, c_void_p, c_void_p, c_void_p]),
    "pdllm_scatter_pages": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int64, c_int, c_int64, c_void_p, c_void_p, c_void_p]),
    "pdllm_copy_pages": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int64, c_int, c_int64, c_int64, c_void_p, c_void_p]),
    "pdllm_enable_peer_access": (c_int, [c_int, c_int]),
    "pdllm_compact_pages_per_head": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
                                             c_int, c_int, c_int64, c_void_p, c_void_p, c_void_p]),
    "pdllm_add_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64, c_int64, c_int64, c_float, c_int, c_void_p]),
    "pdllm_rope_inplace": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int64, c_int, c_void_p]),
    "pdllm_rope_store": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64,
                                 c_int, c_int, c_void_p, c_void_p]),
    "pdllm_silu_mul": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int64, c_int64, c_int, c_void_p]),
    "pdllm_linear_workspace_bytes": (c_int64, [c_int64, c_int64, c_int64]),
    "pdllm_linear": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
                             c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "pdllm_rope_pages": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int64,
                                 c_void_p, c_void_p]),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)

_lib = None
_lock = threading.Lock()


class PdllmError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"pdllm_b200 error {code}: {message}")
        self.code = code


def load() -> ctypes.CDLL:
    """Load the shared library (once) and attach argument types. Raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python prefilling-dllm_b200/build.py` "
                "(or __graft_entry__.build()); there is no fallback path"
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.pdllm_abi_version() != ABI_VERSION:
            raise ImportError(f"{LIB_PATH} has ABI version {lib.pdllm_abi_version()}, expected {ABI_VERSION}")
        _lib = lib
    return _lib


def last_error() -> str:
    msg = load().pdllm_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def check(code: int) -> None:
    """Map a C-ABI return code onto the exception types the reference's Python ops raise."""
    if code == 0:
        return
    msg = last_error()
    if code == E_INVALID:
        raise ValueError(msg)
    if code == E_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise PdllmError(code, msg)
