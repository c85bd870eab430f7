"""Host-side planning of the tcgen05 attention launch, read through the size query of the C-ABI
(`pdllm_attn_workspace_bytes`): no kernel runs, the pointers are placeholders that are never dereferenced. Without a
GPU the planner assumes 148 SMs."""

from ctypes import byref, c_void_p

import pytest

from prefilling_dllm_b200 import _lib

PARTIAL = (128 * 128 + 2 * 128) * 4     # one split-KV partial of one query tile: O [128 x 128] fp32 + (m, l)
HEADER = 64 * 1024                      # arrival counters


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def _params(num_seqs, hq, hkv, max_q, max_seq, num_splits=0, dtype=1):
    p = _lib.AttnParams()
    fake = c_void_p(1 << 20)
    p.q = p.k_new = p.v_new = p.out = p.k_cache = p.v_cache = fake
    p.block_table = p.cu_seqlens_q = p.seq_lens = fake
    p.num_seqs, p.num_q_heads, p.num_kv_heads, p.head_dim = num_seqs, hq, hkv, 128
    p.page_size, p.kv_layout, p.dtype, p.mask_mode = 256, 1, dtype, 0
    p.max_query_len, p.max_seq_len, p.num_splits = max_q, max_seq, num_splits
    p.total_q, p.num_pages, p.max_pages = num_seqs * max_q, 4096, 64
    p.q_stride = p.out_stride = hq * 128
    p.k_stride = p.v_stride = hkv * 128
    p.sm_scale = 0.088
    return p


def _partials(lib, *args, **kwargs):
    n = lib.pdllm_attn_workspace_bytes(byref(_params(*args, **kwargs)))
    assert n >= 0, lib.pdllm_last_error()
    if n == 0:
        return 0
    assert (n - HEADER) % PARTIAL == 0
    return (n - HEADER) // PARTIAL


def test_op_config_two_uneven_splits(lib):
    # 8 requests x 4 KV heads x 3 query-tile pairs = 96 units on 148 SMs: every unit cut in two; 6 tiles per (request, head)
    assert _partials(lib, 8, 28, 4, 96, 4096 + 96) == 8 * 4 * 6 * 2


def test_one_unit_per_sm_runs_unsplit(lib):
    # 37 x 4 = 148 units of two query tiles: one whole wave, nothing to merge
    assert _partials(lib, 37, 28, 4, 36, 4096 + 36) == 0


def test_forced_splits_are_honoured(lib):
    assert _partials(lib, 2, 28, 4, 36, 4096 + 36, num_splits=3) == 2 * 4 * 2 * 3


def test_few_units_go_to_the_cluster_kernel(lib, monkeypatch):
    # one request, one block of 32 rows (two query tiles x 4 KV heads = 8 units): the few-rows kernel cuts every unit into a
    # cluster of up to 16 CTAs, each leaving one share (O, m, l of one query tile) in the workspace ...
    assert _partials(lib, 1, 28, 4, 32, 4161 + 32) == 8 * 16
    # ... a forced split count keeps the shape on the twin-tile kernel, which merges through partials in the workspace
    assert _partials(lib, 1, 28, 4, 32, 4161 + 32, num_splits=12) == 1 * 4 * 2 * 12
    # ... and with the few-rows kernel switched off its cost model settles between 8 and 16 splits
    monkeypatch.setenv("PDLLM_NO_DECODE_KERNEL", "1")
    n = _partials(lib, 1, 28, 4, 32, 4161 + 32)
    assert n % 8 == 0 and 8 <= n // 8 <= 16


def test_whole_waves_then_a_split_tail(lib):
    # 160 units of two query tiles, 17 key tiles: 148 run unsplit, the last 12 (24 query tiles) are cut in four
    assert _partials(lib, 40, 28, 4, 36, 2048 + 36) == 24 * 4


def test_unsupported_shapes_need_no_workspace(lib):
    p = _params(8, 28, 4, 96, 4192)
    p.head_dim = 64                 # runs on the SIMT kernel
    assert lib.pdllm_attn_workspace_bytes(byref(p)) == 0
