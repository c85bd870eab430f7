"""CPU checks of the C-ABI library: it loads without a GPU, exports every symbol the header declares, and its
host-side argument validation answers with the documented codes (no kernel is launched here)."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    import __graft_entry__

    __graft_entry__.build()
    from prefilling_dllm_b200 import _lib

    return _lib


def header_symbols():
    with open(os.path.join(ROOT, "include", "pdllm_b200.h")) as handle:
        text = handle.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pdllm_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(lib):
    declared = header_symbols()
    assert len(declared) >= 19
    handle = lib.load()
    for name in declared:
        assert hasattr(handle, name), f"{name} is declared in include/pdllm_b200.h but not exported"
    assert sorted(lib.EXPORTED_SYMBOLS) == declared, "ctypes signature table and header disagree"
    assert handle.pdllm_abi_version() == lib.ABI_VERSION


def test_header_cites_the_reference_for_every_kernel_entry():
    with open(os.path.join(ROOT, "include", "pdllm_b200.h")) as handle:
        text = handle.read()
    for needle in ("kv_cache_kernels.py", "prefix_prefill.py", "chunked_prefill_decoding_unified_kernel.py",
                   "triton_eviction_scorer.py", "fastdllm_parallelcomp.py", "fastdllm_engine.py"):
        assert needle in text


def test_host_side_validation_codes(lib):
    handle = lib.load()
    p = lib.AttnParams()
    p.total_q, p.num_seqs = 4, 1
    assert handle.pdllm_paged_attention(ctypes.byref(p), None) == lib.E_INVALID  # null tensors
    assert "null" in lib.last_error()
    with pytest.raises(ValueError):
        lib.check(lib.E_INVALID)
    with pytest.raises(NotImplementedError):
        lib.check(lib.E_UNSUPPORTED)
    assert handle.pdllm_topk_chunks(None, 2000, 1, 0, None, None, None) == lib.E_INVALID
    assert handle.pdllm_unmask_workspace_bytes(32) == (32 * 27 + 1) * 4
    assert handle.pdllm_evict_workspace_bytes(28, 8, 1033) == 28 * 8 * 1033 * 4
    assert handle.pdllm_unmask_step(None, 0, None, 0, 0, 10, 1, None, 0, 0.9, 0, None, None, None, None, 0, None) == lib.E_INVALID
    # empty work is a no-op success, as in the reference ops
    assert handle.pdllm_store_kvcache_unified(None, None, None, None, None, 0, 512, 512, 512, 2, 0, None, None) == 0


def test_ops_refuse_cpu_tensors(lib):
    import torch

    from prefilling_dllm_b200 import ops

    x = torch.zeros(2, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.store_kvcache_unified_layout(x, x, torch.zeros(1, 256, 4, 128, dtype=torch.bfloat16),
                                         torch.zeros(1, 256, 4, 128, dtype=torch.bfloat16), torch.zeros(2, dtype=torch.int32))
    with pytest.raises(ValueError, match="CUDA"):
        ops.paged_attention(x, x, x, x.clone(), cu_seqlens_q=torch.tensor([0, 2], dtype=torch.int32), max_query_len=2)


def test_missing_library_fails_loudly(lib, monkeypatch):
    monkeypatch.setattr(lib, "_lib", None)
    monkeypatch.setattr(lib, "LIB_PATH", os.path.join(ROOT, "does-not-exist.so"))
    with pytest.raises(ImportError, match="no fallback"):
        lib.load()
