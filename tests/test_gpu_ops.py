"""Parity of every CUDA op (called through the C-ABI via prefilling_dllm_b200.ops) against the CPU oracle.

Integer / index outputs must be bit-exact; fp32 reductions within 1e-5 relative; bf16 attention within the
1e-2 relative error the north star states (measured as ||out-ref||_F / ||ref||_F, plus a max-abs guard).
"""

import math

import pytest
import torch

from oracle import hotpath as oracle

pytestmark = pytest.mark.gpu

ATTN_REL_TOL = 1e-2  # bf16 attention outputs, relative Frobenius error


@pytest.fixture(scope="module")
def ops(cuda_device):
    from prefilling_dllm_b200 import ops as _ops

    return _ops


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


def row_rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """Worst (token, head) row: max_r ||a_r - b_r|| / ||b_r||. A few bad rows (a mis-masked last tile, one wrong page) vanish in
    a norm over the whole output; they cannot hide here. Rows the reference leaves at zero must be zero."""
    a, b = a.float().cpu(), b.float().cpu()
    num, den = (a - b).norm(dim=-1), b.norm(dim=-1)
    zero = den == 0
    assert float(num[zero].max()) == 0.0 if bool(zero.any()) else True
    return float((num[~zero] / den[~zero]).max())


def assert_attention_close(out: torch.Tensor, ref: torch.Tensor, what=None, tol: float = 1e-2) -> None:
    assert not torch.isnan(out).any(), what
    assert rel_err(out, ref) < tol, what
    assert row_rel_err(out, ref) < tol, what


# ----------------------------------------------------------------------------------------------- (5)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_store_kvcache_unified(ops, cuda_device, dtype):
    g = torch.Generator().manual_seed(1)
    n, hkv, d, pages, page = 300, 4, 128, 6, 256
    key = torch.randn(n, hkv, d, generator=g).to(dtype)
    value = torch.randn(n, hkv, d, generator=g).to(dtype)
    slots = torch.randperm(pages * page, generator=g)[:n].to(torch.int32)
    slots[::7] = -1  # skipped tokens
    k_ref = torch.zeros(pages, page, hkv, d, dtype=dtype)
    v_ref = torch.zeros_like(k_ref)
    oracle.store_kvcache_unified(key, value, k_ref, v_ref, slots)
    k_c = torch.zeros_like(k_ref, device=cuda_device)
    v_c = torch.zeros_like(k_c)
    ops.store_kvcache_unified_layout(key.to(cuda_device), value.to(cuda_device), k_c, v_c, slots.to(cuda_device), "diffusion_lm")
    ops.check_status(cuda_device)
    assert torch.equal(k_c.cpu(), k_ref) and torch.equal(v_c.cpu(), v_ref)


def test_store_kvcache_unified_strided_rows_and_bad_slot(ops, cuda_device):
    g = torch.Generator().manual_seed(2)
    n, hkv, d = 33, 2, 64
    qkv = torch.randn(n, 3 * hkv * d, generator=g).bfloat16().to(cuda_device)
    key = qkv[:, hkv * d:2 * hkv * d].view(n, hkv, d)      # row stride 3*Hkv*D: the fused-QKV case
    value = qkv[:, 2 * hkv * d:].view(n, hkv, d)
    slots = torch.arange(n, dtype=torch.int32)
    k_c = torch.zeros(1, 64, hkv, d, dtype=torch.bfloat16, device=cuda_device)
    v_c = torch.zeros_like(k_c)
    ops.store_kvcache_unified_layout(key, value, k_c, v_c, slots.to(cuda_device), "diffusion_lm")
    ops.check_status(cuda_device)
    assert torch.equal(k_c.view(-1, hkv, d)[:n], key) and torch.equal(v_c.view(-1, hkv, d)[:n], value)
    bad = slots.clone()
    bad[5] = 64 * 1 + 3  # beyond the pool: must be skipped and flagged, not written
    ops.store_kvcache_unified_layout(key, value, k_c, v_c, bad.to(cuda_device), "diffusion_lm")
    with pytest.raises(RuntimeError, match="slot_mapping"):
        ops.check_status(cuda_device)
    assert ops.check_status(cuda_device) == 0  # reading resets the word


def test_store_kvcache_empty(ops, cuda_device):
    key = torch.empty(0, 4, 128, dtype=torch.bfloat16, device=cuda_device)
    cache = torch.zeros(2, 256, 4, 128, dtype=torch.bfloat16, device=cuda_device)
    ops.store_kvcache_unified_layout(key, key.clone(), cache, cache.clone(), torch.empty(0, dtype=torch.int32, device=cuda_device), "diffusion_lm")
    assert float(cache.abs().sum()) == 0.0


def test_store_kvcache_distinct(ops, cuda_device):
    g = torch.Generator().manual_seed(3)
    n, hkv, d, pages, page, x = 200, 4, 128, 3, 256, 8
    key = torch.randn(n, hkv, d, generator=g).bfloat16()
    value = torch.randn(n, hkv, d, generator=g).bfloat16()
    slots = torch.randperm(pages * page, generator=g)[:n].to(torch.int32)
    slots[3] = -1
    k_ref = torch.zeros(pages, hkv, d // x, page, x, dtype=torch.bfloat16)
    v_ref = torch.zeros(pages, hkv, d, page, dtype=torch.bfloat16)
    oracle.store_kvcache_distinct(key, value, k_ref, v_ref, slots)
    k_c, v_c = torch.zeros_like(k_ref, device=cuda_device), torch.zeros_like(v_ref, device=cuda_device)
    ops.store_kvcache_distinct_layout(key.to(cuda_device), value.to(cuda_device), k_c, v_c, slots.to(cuda_device), "diffusion_lm")
    ops.check_status(cuda_device)
    assert torch.equal(k_c.cpu(), k_ref) and torch.equal(v_c.cpu(), v_ref)


class _Ctx:
    pass


def test_load_kvcache_matches_gather(ops, cuda_device):
    g = torch.Generator().manual_seed(4)
    hkv, d, page, pages = 4, 128, 256, 12
    ctx_lens = [300, 0, 512]
    new_lens = [32, 64, 32]
    k_cache = torch.randn(pages, page, hkv, d, generator=g).bfloat16()
    v_cache = torch.randn(pages, page, hkv, d, generator=g).bfloat16()
    bt = torch.tensor([[7, 2, -1], [-1, -1, -1], [0, 11, -1]], dtype=torch.int32)
    cu_q = [0]
    for n in new_lens:
        cu_q.append(cu_q[-1] + n)
    cu_k = [0]
    for c, n in zip(ctx_lens, new_lens):
        cu_k.append(cu_k[-1] + c + n)
    k_new = torch.randn(cu_q[-1], hkv, d, generator=g).bfloat16()
    v_new = torch.randn(cu_q[-1], hkv, d, generator=g).bfloat16()
    k_ref, v_ref = oracle.load_kvcache(k_cache, v_cache, bt, ctx_lens, cu_q, k_new, v_new)
    ctx = _Ctx()
    ctx.block_tables = bt.to(cuda_device)
    ctx.context_lens = torch.tensor(ctx_lens, dtype=torch.int32, device=cuda_device)
    ctx.seq_lens_ts = torch.tensor(new_lens, dtype=torch.int32, device=cuda_device)
    ctx.cu_seqlens_q = torch.tensor(cu_q, dtype=torch.int32, device=cuda_device)
    ctx.cu_seqlens_k = torch.tensor(cu_k, dtype=torch.int32, device=cuda_device)
    k_out, v_out = ops.load_kvcache(k_cache.to(cuda_device), v_cache.to(cuda_device), ctx, k_new.to(cuda_device), v_new.to(cuda_device))
    ops.check_status(cuda_device)
    assert torch.equal(k_out.cpu(), k_ref) and torch.equal(v_out.cpu(), v_ref)


# ----------------------------------------------------------------------------------------------- (3)+(1)
def _attention_case(seed, *, num_seqs, hq, hkv, d, page, chunks_in_pool, pages_per_chunk, sel_chunks, q_lens, dtype,
                    ctx_tail=0, layout="unified"):
    """Build the op-level workload: a pool of chunks per request, sel_chunks picked by a seeded permutation."""
    g = torch.Generator().manual_seed(seed)
    pages_per_req = chunks_in_pool * pages_per_chunk
    num_pages = num_seqs * pages_per_req
    k_cache = torch.randn(num_pages, page, hkv, d, generator=g).to(dtype)
    v_cache = torch.randn(num_pages, page, hkv, d, generator=g).to(dtype)
    bt = torch.full((num_seqs, sel_chunks * pages_per_chunk + 1), -1, dtype=torch.int32)
    seq_lens, cu = [], [0]
    for s in range(num_seqs):
        chosen = torch.randperm(chunks_in_pool, generator=g)[:sel_chunks]
        ids = []
        for c in chosen.tolist():
            ids += [s * pages_per_req + c * pages_per_chunk + i for i in range(pages_per_chunk)]
        bt[s, :len(ids)] = torch.tensor(ids, dtype=torch.int32)
        ctx = len(ids) * page - (ctx_tail if s % 2 == 1 else 0)
        seq_lens.append(ctx + q_lens[s])
        cu.append(cu[-1] + q_lens[s])
    t = cu[-1]
    q = torch.randn(t, hq, d, generator=g).to(dtype)
    k = torch.randn(t, hkv, d, generator=g).to(dtype)
    v = torch.randn(t, hkv, d, generator=g).to(dtype)
    return dict(q=q, k=k, v=v, k_cache=k_cache, v_cache=v_cache, bt=bt, seq_lens=seq_lens, cu=cu)


def _run_attention(ops, dev, case, *, impl, mask=None, bidirectional=True, causal=False, diffusion_blk=32, num_splits=0,
                   with_cache=True, sm_scale=None):
    q, k, v = (case[n].to(dev) for n in ("q", "k", "v"))
    out = torch.full_like(q, float("nan"))
    kwargs = {}
    if with_cache:
        kwargs = dict(key_cache=case["k_cache"].to(dev), value_cache=case["v_cache"].to(dev), block_table=case["bt"].to(dev),
                      seq_lens=torch.tensor(case["seq_lens"], dtype=torch.int32, device=dev), max_seq_len=max(case["seq_lens"]))
    cu = torch.tensor(case["cu"], dtype=torch.int32, device=dev)
    q_lens = [case["cu"][i + 1] - case["cu"][i] for i in range(len(case["cu"]) - 1)]
    used = ops.paged_attention(q, k, v, out, cu_seqlens_q=cu, max_query_len=max(q_lens), sm_scale=sm_scale,
                               mask=None if mask is None else mask.to(dev), causal=causal, bidirectional=bidirectional,
                               diffusion_blk_sz=diffusion_blk, impl=impl, num_splits=num_splits, **kwargs)
    ops.check_status(dev)
    return out, used


def _ref_attention(case, *, mask=None, bidirectional=True, causal=False, diffusion_blk=32, with_cache=True, sm_scale=None):
    return oracle.paged_attention(case["q"], case["k"], case["v"], cu_seqlens_q=case["cu"],
                                  k_cache=case["k_cache"] if with_cache else None, v_cache=case["v_cache"] if with_cache else None,
                                  block_table=case["bt"] if with_cache else None, seq_lens=case["seq_lens"] if with_cache else None,
                                  sm_scale=sm_scale, mask=mask, bidirectional=bidirectional, diffusion_blk=diffusion_blk, causal=causal)


def test_attention_simt_fp32_toy_shape(ops, cuda_device):
    # config "CPU toy": 4 query / 2 KV heads, head_dim 64, fp32
    case = _attention_case(10, num_seqs=2, hq=4, hkv=2, d=64, page=256, chunks_in_pool=4, pages_per_chunk=2, sel_chunks=2,
                           q_lens=[32, 64], dtype=torch.float32, ctx_tail=100)
    out, used = _run_attention(ops, cuda_device, case, impl="auto")
    assert used == "simt"
    ref = _ref_attention(case)
    assert rel_err(out, ref) < 1e-5


@pytest.mark.parametrize("layout", ["unified", "distinct"])
def test_attention_simt_bf16_layouts(ops, cuda_device, layout):
    case = _attention_case(11, num_seqs=3, hq=28, hkv=4, d=128, page=256, chunks_in_pool=3, pages_per_chunk=1, sel_chunks=2,
                           q_lens=[32, 96, 7], dtype=torch.bfloat16, ctx_tail=37)
    ref = _ref_attention(case)
    if layout == "distinct":
        x = 8
        pages, page, hkv, d = case["k_cache"].shape
        kd = case["k_cache"].view(pages, page, hkv, d // x, x).permute(0, 2, 3, 1, 4).contiguous()
        vd = case["v_cache"].permute(0, 2, 3, 1).contiguous()
        ku, vu = oracle.distinct_to_unified(kd, vd)
        assert torch.equal(ku, case["k_cache"]) and torch.equal(vu, case["v_cache"])
        case = dict(case, k_cache=kd, v_cache=vd)
    out, used = _run_attention(ops, cuda_device, case, impl="simt")
    assert used == "simt"
    assert rel_err(out, ref) < ATTN_REL_TOL


def test_attention_simt_masks(ops, cuda_device):
    case = _attention_case(12, num_seqs=2, hq=8, hkv=2, d=64, page=256, chunks_in_pool=2, pages_per_chunk=1, sel_chunks=1,
                           q_lens=[96, 96], dtype=torch.float32)
    g = torch.Generator().manual_seed(5)
    dense = torch.rand(96, 96, generator=g) > 0.3
    dense[5, :] = False  # a row whose new keys are all hidden still sees the context
    for kwargs in (dict(mask=dense, bidirectional=True), dict(bidirectional=False), dict(mask=dense, bidirectional=False),
                   dict(causal=True)):
        out, _ = _run_attention(ops, cuda_device, case, impl="simt", **kwargs)
        assert rel_err(out, _ref_attention(case, **kwargs)) < 1e-5, kwargs
    # no context at all + a fully hidden row → zeros, as the reference kernel produces
    out, _ = _run_attention(ops, cuda_device, case, impl="simt", mask=dense, with_cache=False)
    ref = _ref_attention(case, mask=dense, with_cache=False)
    assert rel_err(out, ref) < 1e-5
    assert float(out[5].abs().max()) == 0.0


def test_attention_tc_small_single_tile(ops, cuda_device):
    # one request, one KV group tile: the smallest shape the tcgen05 kernel takes
    case = _attention_case(20, num_seqs=1, hq=28, hkv=4, d=128, page=256, chunks_in_pool=2, pages_per_chunk=1, sel_chunks=1,
                           q_lens=[16], dtype=torch.bfloat16)
    out, used = _run_attention(ops, cuda_device, case, impl="tc", num_splits=1)
    assert used == "tc"
    assert_attention_close(out, _ref_attention(case))


@pytest.mark.parametrize("num_splits", [1, 3, 0])
def test_attention_tc_ragged_batch(ops, cuda_device, num_splits):
    case = _attention_case(21, num_seqs=3, hq=28, hkv=4, d=128, page=256, chunks_in_pool=4, pages_per_chunk=2, sel_chunks=2,
                           q_lens=[96, 32, 50], dtype=torch.bfloat16, ctx_tail=77)
    out, used = _run_attention(ops, cuda_device, case, impl="tc", num_splits=num_splits)
    assert used == "tc"
    ref = _ref_attention(case)
    assert_attention_close(out, ref)
    assert float((out.float().cpu() - ref).abs().max()) < 0.05


def test_attention_tc_uneven_split_and_fused_merge_ragged(ops, cuda_device):
    """96 (sequence, KV head, tile pair) units on 148 SMs: the plan cuts every unit in two uneven KV splits and the last
    CTA of a pair merges them. Ragged: query lengths from one tile to three, every other context a partial page, so
    some second splits get nothing to attend (neutral partials) and some pairs have an empty second tile."""
    q_lens = [50, 36, 18, 40, 7, 36, 36, 19, 36, 25, 36, 36]          # 12 sequences x 4 KV heads x 2 pairs where q_len > 36
    case = _attention_case(31, num_seqs=12, hq=28, hkv=4, d=128, page=256, chunks_in_pool=4, pages_per_chunk=2, sel_chunks=3,
                           q_lens=q_lens, dtype=torch.bfloat16, ctx_tail=200)     # 13 key tiles: long enough for the uneven cut
    for kwargs in (dict(), dict(causal=True), dict(bidirectional=False)):
        out, used = _run_attention(ops, cuda_device, case, impl="tc", **kwargs)
        assert used == "tc"
        ref = _ref_attention(case, **kwargs)
        assert_attention_close(out, ref, kwargs)
    # twice in a row through the same workspace: the arrival counters must have returned to zero
    again, _ = _run_attention(ops, cuda_device, case, impl="tc")
    first, _ = _run_attention(ops, cuda_device, case, impl="tc")
    assert torch.equal(again, first)


def test_attention_tc_masks_and_prefill(ops, cuda_device):
    case = _attention_case(22, num_seqs=2, hq=28, hkv=4, d=128, page=256, chunks_in_pool=2, pages_per_chunk=1, sel_chunks=1,
                           q_lens=[200, 160], dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(6)
    dense = torch.rand(200, 200, generator=g) > 0.3
    dense[9, :] = False
    for kwargs in (dict(mask=dense, bidirectional=True), dict(bidirectional=False), dict(causal=True),
                   dict(causal=True, with_cache=False), dict(with_cache=False), dict(mask=dense, with_cache=False)):
        out, used = _run_attention(ops, cuda_device, case, impl="tc", **kwargs)
        assert used == "tc"
        assert_attention_close(out, _ref_attention(case, **kwargs), kwargs)


def test_attention_tc_mha_fp16(ops, cuda_device):
    # LLaDA-like: MHA (group 1), fp16 inputs
    case = _attention_case(23, num_seqs=2, hq=8, hkv=8, d=128, page=256, chunks_in_pool=2, pages_per_chunk=2, sel_chunks=1,
                           q_lens=[32, 32], dtype=torch.float16)
    out, used = _run_attention(ops, cuda_device, case, impl="auto")
    assert used == "tc"
    assert rel_err(out, _ref_attention(case)) < ATTN_REL_TOL


@pytest.mark.parametrize("num_splits", [0, 1, 3])
def test_attention_tc_mha_one_query_tile_ragged(ops, cuda_device, num_splits):
    """MHA decode shape: every sequence has at most 128 (token x head) rows per KV head, so every CTA has one query tile
    and its second half idles. Ragged query lengths up to a full tile, contexts of 3 pages or 3 pages minus 250 tokens
    (odd and even numbers of key tiles), every mask mode, splits forced and chosen."""
    q_lens = [32, 7, 128, 64, 1]
    case = _attention_case(41, num_seqs=5, hq=8, hkv=8, d=128, page=256, chunks_in_pool=4, pages_per_chunk=1, sel_chunks=3,
                           q_lens=q_lens, dtype=torch.bfloat16, ctx_tail=250)
    g = torch.Generator().manual_seed(8)
    dense = torch.rand(128, 128, generator=g) > 0.4
    dense[3, :] = False
    for kwargs in (dict(), dict(bidirectional=False), dict(causal=True), dict(mask=dense, bidirectional=True)):
        out, used = _run_attention(ops, cuda_device, case, impl="tc", num_splits=num_splits, **kwargs)
        assert used == "tc"
        ref = _ref_attention(case, **kwargs)
        assert_attention_close(out, ref, kwargs)
    again, _ = _run_attention(ops, cuda_device, case, impl="tc", num_splits=num_splits)
    first, _ = _run_attention(ops, cuda_device, case, impl="tc", num_splits=num_splits)
    assert torch.equal(again, first)


def test_attention_tc_short_contexts_single_key_tile(ops, cuda_device):
    """Contexts of one 128-token page or 68 tokens: CTAs with one or two key tiles, and splits that get none."""
    case = _attention_case(42, num_seqs=3, hq=4, hkv=4, d=128, page=128, chunks_in_pool=2, pages_per_chunk=1, sel_chunks=1,
                           q_lens=[16, 100, 128], dtype=torch.float16, ctx_tail=60)
    for num_splits in (0, 1, 2):
        out, used = _run_attention(ops, cuda_device, case, impl="tc", num_splits=num_splits)
        assert used == "tc"
        assert rel_err(out, _ref_attention(case)) < ATTN_REL_TOL, num_splits


def test_attention_tc_whole_waves_then_split_tail(ops, cuda_device):
    """160 (sequence, KV head) units of 17 key tiles on 148 SMs: the plan runs 148 units unsplit in the first wave and
    cuts the last 12 in three, so CTAs that write the output directly and CTAs that publish partials share one launch.
    Ragged contexts; repeated launches must agree bit for bit (the arrival counters return to zero)."""
    q_lens = [32, 20, 32, 32, 5, 32, 32, 32, 17, 32]
    case = _attention_case(43, num_seqs=10, hq=16, hkv=16, d=128, page=256, chunks_in_pool=2, pages_per_chunk=4, sel_chunks=2,
                           q_lens=q_lens, dtype=torch.bfloat16, ctx_tail=300)
    for kwargs in (dict(), dict(bidirectional=False)):
        out, used = _run_attention(ops, cuda_device, case, impl="tc", **kwargs)
        assert used == "tc"
        ref = _ref_attention(case, **kwargs)
        assert_attention_close(out, ref, kwargs)
    again, _ = _run_attention(ops, cuda_device, case, impl="tc")
    first, _ = _run_attention(ops, cuda_device, case, impl="tc")
    assert torch.equal(again, first)


def test_attention_tc_shapes_the_runtime_issues(ops, cuda_device):
    """The shapes a Dream-7B-sized request really sends to the tensor-core kernel (28 / 4 heads, d 128, bf16):
    the scoring forward — 8 packed causal rows of 1093 tokens, no cache; the joint prefill — one bidirectional sequence of
    4193 tokens, no cache (its page write comes after attention); a denoise block — 96 and 32 new rows over a 17-page
    table whose last page holds 65 tokens. Checked row by row."""
    scoring = _attention_case(51, num_seqs=8, hq=28, hkv=4, d=128, page=256, chunks_in_pool=1, pages_per_chunk=1, sel_chunks=1,
                              q_lens=[1093] * 8, dtype=torch.bfloat16)
    out, used = _run_attention(ops, cuda_device, scoring, impl="auto", causal=True, with_cache=False)
    assert used == "tc"
    assert_attention_close(out, _ref_attention(scoring, causal=True, with_cache=False), "causal 8 x 1093")
    joint = _attention_case(52, num_seqs=1, hq=28, hkv=4, d=128, page=256, chunks_in_pool=1, pages_per_chunk=1, sel_chunks=1,
                            q_lens=[4193], dtype=torch.bfloat16)
    out, used = _run_attention(ops, cuda_device, joint, impl="auto", with_cache=False)
    assert used == "tc"
    assert_attention_close(out, _ref_attention(joint, with_cache=False), "bidirectional 4193")
    block = _attention_case(53, num_seqs=2, hq=28, hkv=4, d=128, page=256, chunks_in_pool=17, pages_per_chunk=1, sel_chunks=17,
                            q_lens=[32, 96], dtype=torch.bfloat16, ctx_tail=256 - 65)
    assert block["seq_lens"] == [17 * 256 + 32, 16 * 256 + 65 + 96]
    out, used = _run_attention(ops, cuda_device, block, impl="auto")
    assert used == "tc"
    assert_attention_close(out, _ref_attention(block), "decode rows over a ragged 17-page table")


def test_attention_few_rows_cluster_kernel(ops, cuda_device):
    """A block of decode rows of one or a few requests: one query tile per CTA, the KV splits of a (sequence, KV head, query
    tile) merged inside a thread-block cluster through distributed shared memory. Ragged query lengths and contexts (a last
    page of 65 tokens, splits that get nothing), GQA 7 and MHA, every mask rule, poisoned page tails; checked row by row
    against the oracle and, bit for bit, against a second launch."""
    g = torch.Generator().manual_seed(9)
    dense = torch.rand(64, 64, generator=g) > 0.4
    dense[3, :] = False
    shapes = [
        dict(num_seqs=1, hq=28, hkv=4, q_lens=[32], sel_chunks=17, ctx_tail=0),                     # one request's denoise step
        dict(num_seqs=2, hq=28, hkv=4, q_lens=[32, 32], sel_chunks=17, ctx_tail=256 - 65),          # the second ends in a 65-token page
        dict(num_seqs=3, hq=28, hkv=4, q_lens=[32, 7, 20], sel_chunks=5, ctx_tail=100),
        dict(num_seqs=2, hq=8, hkv=8, q_lens=[32, 64], sel_chunks=3, ctx_tail=250),                 # MHA: 32 and 64 rows per tile
        dict(num_seqs=1, hq=28, hkv=4, q_lens=[4], sel_chunks=2, ctx_tail=0),                       # a draft round
    ]
    for i, sh in enumerate(shapes):
        case = _attention_case(60 + i, num_seqs=sh["num_seqs"], hq=sh["hq"], hkv=sh["hkv"], d=128, page=256, chunks_in_pool=sh["sel_chunks"],
                               pages_per_chunk=1, sel_chunks=sh["sel_chunks"], q_lens=sh["q_lens"], dtype=torch.bfloat16, ctx_tail=sh["ctx_tail"])
        # rows of every page past what any sequence reads hold NaN bit patterns: they must not leak through masked keys
        for s_idx in range(sh["num_seqs"]):
            ctx = case["seq_lens"][s_idx] - sh["q_lens"][s_idx]
            last_page, used = int(case["bt"][s_idx, (ctx - 1) // 256]), (ctx - 1) % 256 + 1
            if used < 256:
                case["k_cache"][last_page, used:] = float("nan")
                case["v_cache"][last_page, used:] = float("nan")
        for kwargs in (dict(), dict(bidirectional=False), dict(causal=True), dict(mask=dense, bidirectional=True)):
            if "mask" in kwargs and max(sh["q_lens"]) > 64:
                continue
            out, used = _run_attention(ops, cuda_device, case, impl="auto", **kwargs)
            assert used == "tc" and ops.LAST_ATTENTION_USED_CLUSTERS, (sh, kwargs)
            clean = dict(case, k_cache=torch.nan_to_num(case["k_cache"]), v_cache=torch.nan_to_num(case["v_cache"]))
            assert_attention_close(out, _ref_attention(clean, **kwargs), (sh, kwargs))
            again, _ = _run_attention(ops, cuda_device, case, impl="auto", **kwargs)
            assert torch.equal(out, again), (sh, kwargs)


def test_attention_tc_uninitialised_pool_tail_is_harmless(ops, cuda_device):
    # rows of a page past the context length may hold NaN bit patterns; they must not leak into the output
    case = _attention_case(24, num_seqs=2, hq=28, hkv=4, d=128, page=256, chunks_in_pool=2, pages_per_chunk=1, sel_chunks=1,
                           q_lens=[32, 32], dtype=torch.bfloat16, ctx_tail=100)
    ref = _ref_attention(case)
    poisoned = dict(case)
    kc, vc = case["k_cache"].clone(), case["v_cache"].clone()
    page = int(case["bt"][1, 0])
    kc[page, 156:] = float("nan")
    vc[page, 156:] = float("nan")
    poisoned["k_cache"], poisoned["v_cache"] = kc, vc
    for impl in ("tc", "simt"):
        out, _ = _run_attention(ops, cuda_device, poisoned, impl=impl)
        assert not torch.isnan(out).any(), impl
        assert rel_err(out, ref) < ATTN_REL_TOL, impl


def test_attention_op_level_config_full_size(ops, cuda_device):
    """The op-level decode-attention shape at full size: 8 requests, 28/4 heads, d 128, page 256, pool of 32 chunks x 1024 tokens per request,
    4 chunks picked by a seeded permutation, 64 query + 32 response rows, bidirectional."""
    case = _attention_case(0, num_seqs=8, hq=28, hkv=4, d=128, page=256, chunks_in_pool=32, pages_per_chunk=4, sel_chunks=4,
                           q_lens=[96] * 8, dtype=torch.bfloat16)
    out, used = _run_attention(ops, cuda_device, case, impl="auto")
    assert used == "tc"
    ref = _ref_attention(case)
    assert_attention_close(out, ref)
    # the SIMT kernel is an independent on-device witness of the same answer
    out_simt, _ = _run_attention(ops, cuda_device, case, impl="simt")
    assert rel_err(out_simt, ref) < ATTN_REL_TOL
    # linearity in V: attention(q, k, 2v) == 2 attention(q, k, v) exactly in bf16 (power-of-two scaling)
    doubled = dict(case, v=case["v"] * 2, v_cache=case["v_cache"] * 2)
    out2, _ = _run_attention(ops, cuda_device, doubled, impl="auto")
    assert torch.equal(out2.float(), out.float() * 2)


def test_flash_decoding_shim_reference_signature(ops, cuda_device):
    case = _attention_case(25, num_seqs=1, hq=28, hkv=4, d=128, page=256, chunks_in_pool=2, pages_per_chunk=2, sel_chunks=2,
                           q_lens=[32], dtype=torch.bfloat16)
    dev = cuda_device
    q, k, v = (case[n].to(dev) for n in ("q", "k", "v"))
    out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(128)
    ops.diffusion_lm_parallel_flash_decoding(
        q, k, v, out, "auto", case["k_cache"].to(dev), case["v_cache"].to(dev), case["bt"].to(dev),
        torch.tensor(case["cu"], dtype=torch.int32, device=dev), torch.tensor(case["seq_lens"], dtype=torch.int32, device=dev),
        max(case["seq_lens"]), 32, 1.0, 1.0, 32, None, None, scale, torch.ones(32, 32, dtype=torch.bool, device=dev))
    ops.check_status(dev)
    # bidirectional defaults to False: with a 32-row block and BLOCK_M = 64 every new key is still visible
    assert rel_err(out, _ref_attention(case, bidirectional=False, sm_scale=scale)) < ATTN_REL_TOL
    with pytest.raises(NotImplementedError):
        ops.diffusion_lm_parallel_flash_decoding(q, k, v, out, "fp8_e4m3", case["k_cache"].to(dev), case["v_cache"].to(dev),
                                                 case["bt"].to(dev), torch.tensor(case["cu"], dtype=torch.int32, device=dev),
                                                 torch.tensor(case["seq_lens"], dtype=torch.int32, device=dev), 0, 32, 1.0, 1.0)


# ----------------------------------------------------------------------------------------------- (4)
def _peaked_logits(g, rows, vocab, peaks):
    """rows x vocab logits whose max softmax probability is (about) peaks[r]."""
    logits = torch.randn(rows, vocab, generator=g) * 0.1
    for r, p in enumerate(peaks):
        if p is None:
            continue
        # one dominant logit: p = e^a / (e^a + sum_rest)
        rest = torch.logsumexp(torch.cat([logits[r, :7], logits[r, 8:]]), dim=0)
        logits[r, 7] = rest + math.log(p / (1 - p))
    return logits


@pytest.mark.parametrize("mode", ["engine_fp32", "eval_bf16", "eval_fp32", "llada_noshift"])
def test_unmask_step_matches_reference_rule(ops, cuda_device, mode):
    g = torch.Generator().manual_seed(30)
    block_len, vocab, mask_id = 32, 4099, 4098
    peaks = [None] * block_len
    for r, p in ((3, 0.95), (4, 0.9001), (5, 0.8999), (6, 0.9), (9, 0.5), (12, 0.999)):
        peaks[r] = p
    logits = _peaked_logits(g, block_len, vocab, peaks)
    last = torch.randn(vocab, generator=g)
    dtype = torch.bfloat16 if mode == "eval_bf16" else torch.float32
    softmax_dtype = torch.float32 if mode == "engine_fp32" else None
    shift = mode != "llada_noshift"
    logits, last = logits.to(dtype), last.to(dtype)
    ids = torch.full((block_len,), mask_id, dtype=torch.int64)
    ids[0] = 11
    ids[20:24] = torch.tensor([5, 6, 7, 8])
    ref_ids, ref_conf, ref_x0 = oracle.unmask_step(logits, ids, mask_token_id=mask_id, threshold=0.9, last_logit=last, shift=shift,
                                                   softmax_dtype=softmax_dtype)
    dev_ids = ids.to(cuda_device)
    counts, conf, x0 = ops.unmask_step(logits.to(cuda_device), dev_ids, mask_token_id=mask_id, threshold=0.9,
                                       last_logit=last.to(cuda_device), shift=shift, softmax_dtype=softmax_dtype, return_details=True)
    assert torch.equal(dev_ids.cpu(), ref_ids)
    assert torch.equal(x0.cpu(), ref_x0)
    finite = torch.isfinite(ref_conf.float())
    assert torch.allclose(conf.cpu()[finite], ref_conf.float()[finite], rtol=2e-6 if dtype == torch.float32 else 0, atol=0)
    before = int((ids == mask_id).sum())
    after = int((ref_ids == mask_id).sum())
    assert counts.cpu().tolist() == [before, before - after, after]
    assert before - after >= 2  # the threshold branch fired, not only the always-accepted top slot


@pytest.mark.parametrize("mode", ["engine_fp32", "eval_bf16", "llada_noshift"])
def test_unmask_step_batched_equals_per_request_steps(ops, cuda_device, mode):
    """Several requests in one launch: each block must come out exactly as the oracle's single-request step gives it,
    with its own last logit, its own ids and its own counts; repeated steps reuse the (self-clearing) workspace."""
    g = torch.Generator().manual_seed(33)
    batch, block_len, vocab, mask_id = 5, 32, 4099, 4098
    dtype = torch.bfloat16 if mode == "eval_bf16" else torch.float32
    softmax_dtype = torch.float32 if mode == "engine_fp32" else None
    shift = mode != "llada_noshift"
    logits = torch.stack([_peaked_logits(g, block_len, vocab, [0.95 if (r + b) % 5 == 0 else None for r in range(block_len)])
                          for b in range(batch)]).to(dtype)
    last = torch.randn(batch, vocab, generator=g).to(dtype)
    ids = torch.full((batch, block_len), mask_id, dtype=torch.int64)
    ids[:, 0] = torch.arange(batch) + 3
    ids[2, 10:20] = 7                   # a partly filled block
    ids[4, :] = 9                       # a finished block: no candidates
    dev_ids = ids.to(cuda_device)
    dev_logits, dev_last = logits.to(cuda_device), last.to(cuda_device)
    ref = ids.clone()
    for step in range(3):
        counts = ops.unmask_step_batched(dev_logits, dev_ids, mask_token_id=mask_id, threshold=0.9, last_logit=dev_last if shift else None,
                                         shift=shift, softmax_dtype=softmax_dtype)
        for b in range(batch):
            before = int((ref[b] == mask_id).sum())
            ref[b], _, _ = oracle.unmask_step(logits[b], ref[b], mask_token_id=mask_id, threshold=0.9, last_logit=last[b] if shift else None,
                                              shift=shift, softmax_dtype=softmax_dtype)
            after = int((ref[b] == mask_id).sum())
            assert counts[b].cpu().tolist() == [before, before - after, after], (step, b)
        assert torch.equal(dev_ids.cpu(), ref), step
    ops.check_status(cuda_device)


def test_unmask_step_flat_logits_make_exactly_one_step(ops, cuda_device):
    # random-init models: max probability ~ 1/V, so exactly the most confident slot is filled each step
    g = torch.Generator().manual_seed(31)
    block_len, vocab, mask_id = 32, 152064, 151666
    logits = (torch.randn(block_len, vocab, generator=g) * 1.2).bfloat16()
    ids = torch.full((block_len,), mask_id, dtype=torch.int64)
    ids[0] = 42
    dev_ids, dev_logits = ids.to(cuda_device), logits.to(cuda_device)
    steps = 0
    ref = ids.clone()
    while bool((ref == mask_id).any()):
        ref, _, _ = oracle.unmask_step(logits, ref, mask_token_id=mask_id, threshold=0.9, last_logit=None, shift=True, softmax_dtype=torch.float32)
        counts = ops.unmask_step(dev_logits, dev_ids, mask_token_id=mask_id, threshold=0.9, shift=True, softmax_dtype=torch.float32)
        steps += 1
        assert torch.equal(dev_ids.cpu(), ref), steps
        assert counts.cpu().tolist()[1] == 1
    assert steps == 31
    # nothing left to fill: a further call is a no-op and reports zero candidates
    counts = ops.unmask_step(dev_logits, dev_ids, mask_token_id=mask_id, threshold=0.9)
    assert counts.cpu().tolist() == [0, 0, 0] and torch.equal(dev_ids.cpu(), ref)


# ----------------------------------------------------------------------------------------------- (2a)(2b)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_self_information_scores(ops, cuda_device, dtype):
    g = torch.Generator().manual_seed(40)
    n_chunks, n_labels, vocab = 8, 34, 1024 if dtype == torch.float32 else 152064
    rows = (torch.randn(n_chunks, n_labels, vocab, generator=g) * 1.3).to(dtype)
    labels = torch.randint(0, vocab, (n_labels,), generator=g)
    ref_scores, ref_nll = oracle.self_information_scores(rows, labels)
    scores, nll = ops.self_information_scores(rows.view(-1, vocab).to(cuda_device), labels.to(cuda_device), n_chunks, return_nll=True)
    ops.check_status(cuda_device)
    assert torch.allclose(nll.cpu(), ref_nll, rtol=1e-5, atol=1e-5)
    assert torch.allclose(scores.cpu(), ref_scores, rtol=1e-5, atol=1e-5)
    # the ranking the scores feed is identical
    sel, cnt = ops.topk_chunks(scores, 4)
    assert sel.cpu()[: int(cnt.item())].tolist() == oracle.rank_chunks(ref_scores.tolist(), 4)


def test_self_information_bad_label_is_flagged(ops, cuda_device):
    rows = torch.zeros(2, 16, dtype=torch.float32, device=cuda_device)
    labels = torch.tensor([99], dtype=torch.int64, device=cuda_device)
    scores = ops.self_information_scores(rows, labels, 2)
    assert scores.cpu().tolist() == [float("-inf")] * 2
    with pytest.raises(RuntimeError, match="label"):
        ops.check_status(cuda_device)


def test_topk_chunks_stable_ties_and_edges(ops, cuda_device):
    cases = [
        ([0.5, 0.7, 0.7, 0.1, 0.7, float("nan"), float("inf"), -1.0], 3, False),
        ([0.5, 0.7, 0.7, 0.1, 0.7, 0.2, 0.3, -1.0], 2, True),
        ([1.0, 1.0, 1.0, 1.0], 2, False),
        ([3.0, 2.0, 1.0], 0, False),
        ([3.0, 2.0, 1.0], 10, False),
        ([float("-inf")] * 5, 2, False),
        ([-6.93 + 1e-6 * ((i * 7919) % 13) for i in range(32)], 8, False),
    ]
    for scores, k, keep_first in cases:
        t = torch.tensor(scores, dtype=torch.float32)
        sel, cnt = ops.topk_chunks(t.to(cuda_device), k, keep_first)
        expect = oracle.rank_chunks(t.tolist(), k, keep_first)
        assert sel.cpu()[: int(cnt.item())].tolist() == expect, (scores, k, keep_first)
    sel, cnt = ops.topk_chunks(torch.empty(0, dtype=torch.float32, device=cuda_device), 4)
    assert int(cnt.item()) == 0


# ----------------------------------------------------------------------------------------------- (2c)
@pytest.mark.parametrize("dtype,hq,hkv,d", [(torch.float32, 4, 2, 64), (torch.bfloat16, 28, 4, 128)])
def test_query_to_chunk_scores(ops, cuda_device, dtype, hq, hkv, d):
    g = torch.Generator().manual_seed(50)
    prefix, chunk, w = 1, 700, 8
    length = prefix + chunk + w
    q = torch.randn(length, hq, d, generator=g).to(dtype)
    k = torch.randn(length, hkv, d, generator=g).to(dtype)
    scale = d ** -0.5
    for mask, reduce in (("causal", "sum"), ("full", "mean")):
        ref = oracle.query_to_chunk_scores(q, k, prefix_len=prefix, chunk_len=chunk, query_len=w, scale=scale, reduce_mode=reduce,
                                           causal=mask == "causal")
        out = ops.query_to_chunk_attention_scores(q.to(cuda_device), k.to(cuda_device), prefix_len=prefix, chunk_len=chunk, query_len=w,
                                                  scale=scale, reduce_mode=reduce, attention_mask=mask)
        assert out.shape == (hq, chunk) and out.dtype == torch.float32
        assert torch.allclose(out.cpu(), ref, rtol=2e-4, atol=1e-7), (mask, reduce)


def test_query_to_chunk_scores_error_behaviour(ops, cuda_device):
    q = torch.randn(20, 4, 64)
    with pytest.raises(ValueError, match="CUDA"):
        ops.query_to_chunk_attention_scores(q, q[:, :2], prefix_len=1, chunk_len=10, query_len=8, scale=1.0)
    qc = q.to(cuda_device)
    with pytest.raises(ValueError, match="too large"):
        ops.query_to_chunk_attention_scores(qc.repeat(8, 1, 1), qc.repeat(8, 1, 1)[:, :2], prefix_len=1, chunk_len=10, query_len=65, scale=1.0)
    assert ops.query_to_chunk_attention_scores(qc, qc[:, :2], prefix_len=1, chunk_len=0, query_len=8, scale=1.0).numel() == 0


@pytest.mark.parametrize("per_head", [False, True])
def test_evict_select_matches_reference_rule(ops, cuda_device, per_head):
    g = torch.Generator().manual_seed(60)
    n_layers, hq, hkv, chunk, cap = 2, 4, 2, 512, 129
    scores = torch.rand(n_layers, hq, chunk, generator=g)
    scores[:, :, 100:140] = 0.0  # a flat stretch: max-pool plateaus and exact ties
    if per_head:
        pooled_ref = torch.stack([oracle.per_head_token_scores(scores[l], hkv) for l in range(n_layers)])
        keep_ref = torch.stack([torch.stack([oracle.select_positions_from_token_scores(pooled_ref[l, h], capacity=cap, chunk_len=chunk)
                                             for h in range(hkv)]) for l in range(n_layers)])
    else:
        pooled_ref = oracle.global_token_scores([scores[l] for l in range(n_layers)]).unsqueeze(0)
        keep_ref = oracle.select_positions_from_token_scores(pooled_ref[0], capacity=cap, chunk_len=chunk).unsqueeze(0)
    keep, pooled = ops.evict_select(scores.to(cuda_device), num_kv_heads=hkv, keep_count=cap, per_head=per_head, return_pooled=True)
    assert torch.allclose(pooled.cpu(), pooled_ref, rtol=1e-6, atol=1e-7)
    # rank on the device's own pooled values so that ulp-level reduction-order differences cannot move the cut
    if per_head:
        keep_dev_rule = torch.stack([torch.stack([oracle.select_positions_from_token_scores(pooled.cpu()[l, h], capacity=cap, chunk_len=chunk)
                                                  for h in range(hkv)]) for l in range(n_layers)])
    else:
        keep_dev_rule = oracle.select_positions_from_token_scores(pooled.cpu()[0], capacity=cap, chunk_len=chunk).unsqueeze(0)
    assert torch.equal(keep.cpu(), keep_dev_rule)
    assert torch.equal(keep.cpu(), keep_ref)
    assert bool((keep.cpu()[..., 0] == 0).all())                       # chunk BOS always kept
    assert bool((keep.cpu()[..., 1:] > keep.cpu()[..., :-1]).all())    # ascending, no duplicates


def test_evict_select_low_and_no_bos(ops, cuda_device):
    g = torch.Generator().manual_seed(61)
    scores = torch.rand(1, 2, 64, generator=g)
    pooled = oracle.global_token_scores([scores[0]], pooling="none")
    for keep_high, force in ((False, True), (True, False), (False, False)):
        ref = oracle.select_positions_from_token_scores(pooled, capacity=10, chunk_len=64, keep_high=keep_high, force_keep_first=force)
        keep = ops.evict_select(scores.to(cuda_device), num_kv_heads=2, keep_count=10, pool_kernel=1, force_keep_first=force, keep_high=keep_high)
        assert keep.cpu()[0].tolist() == ref.tolist()
    # capacity >= chunk: everything is kept
    keep = ops.evict_select(scores.to(cuda_device), num_kv_heads=2, keep_count=64)
    assert keep.cpu()[0].tolist() == list(range(64))


# ----------------------------------------------------------------------------------------------- PD boundary
def test_gather_scatter_compact_pages(ops, cuda_device):
    g = torch.Generator().manual_seed(70)
    pages, page, hkv, d = 10, 256, 4, 128
    cache = torch.randn(pages, page, hkv, d, generator=g).bfloat16()
    page_ids = [7, 2, 9]
    n_tokens = 2 * page + 57
    dense_ref = torch.cat([cache[p] for p in page_ids])[:n_tokens]
    dev_cache = cache.to(cuda_device)
    dense = ops.gather_pages(dev_cache, page_ids, n_tokens)
    assert torch.equal(dense.cpu(), dense_ref)
    # scatter into other pages of another pool and read back
    pool2 = torch.zeros_like(dev_cache)
    ops.scatter_pages(dense, pool2, [1, 4, 5])
    assert torch.equal(ops.gather_pages(pool2, [1, 4, 5], n_tokens).cpu(), dense_ref)
    # per-head compaction in place to the front of the same pages
    keep = torch.stack([torch.sort(torch.randperm(n_tokens, generator=g)[:300]).values for _ in range(hkv)])
    ref = oracle.compact_per_head(dense_ref, keep)
    ops.compact_pages_per_head(dev_cache, page_ids, page_ids, keep.to(cuda_device), src_tokens=n_tokens)
    ops.check_status(cuda_device)
    assert torch.equal(ops.gather_pages(dev_cache, page_ids, 300).cpu(), ref)
    with pytest.raises(ValueError):
        ops.gather_pages(dev_cache, [1], 2 * page)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_pages_in_place(ops, cuda_device, dtype):
    """K rows stored un-rotated, rotated in place afterwards == the eager `k * cos + rotate_half(k) * sin` (bit-exact:
    the kernel rounds each product and the sum to the cache dtype like the eager expression does)."""
    g = torch.Generator().manual_seed(71)
    pages, page, hkv, d = 6, 128, 2, 128
    cache = torch.randn(pages, page, hkv, d, generator=g).to(dtype)
    page_ids = [4, 1, 3]
    start, n = 100, 200                       # crosses two page boundaries
    positions = torch.randint(0, 40000, (n,), generator=g)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, d, 2).float() / d))
    freqs = positions.float().unsqueeze(-1) * inv_freq
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    dense = torch.cat([cache[p] for p in page_ids])
    rows = dense[start:start + n]
    rot = torch.cat((-rows[..., d // 2:], rows[..., : d // 2]), dim=-1)
    expect = dense.clone()
    expect[start:start + n] = rows * cos.unsqueeze(1) + rot * sin.unsqueeze(1)
    dev_cache = cache.to(cuda_device)
    ops.rope_pages(dev_cache, page_ids, start, cos.to(cuda_device), sin.to(cuda_device))
    ops.check_status(cuda_device)
    got = ops.gather_pages(dev_cache, page_ids, 3 * page).cpu()
    assert torch.equal(got, expect)
    untouched = [p for p in range(pages) if p not in page_ids]
    assert torch.equal(dev_cache.cpu()[untouched], cache[untouched])
    with pytest.raises(ValueError):
        ops.rope_pages(dev_cache, [0], 0, cos.to(cuda_device), sin.to(cuda_device))


@pytest.mark.parametrize("hidden,rows", [(3584, 32), (4096, 5), (8192, 3), (520, 9), (8200, 2)])
def test_add_rmsnorm_one_vector_per_thread(ops, cuda_device, hidden, rows):
    """16-bit rows of up to 8192 elements take the one-pass kernel (a 16-byte vector per thread, ragged last warp at 520);
    8200 is past it and takes the loop kernel. Same gates as against eager: the residual row bit-exact, the normed row equal
    but for stray last bits from the order of the fp32 sum."""
    g = torch.Generator().manual_seed(hidden + rows)
    for dtype in (torch.bfloat16, torch.float16):
        x = torch.randn(rows, hidden, generator=g).to(dtype)
        delta = torch.randn(rows, hidden, generator=g).to(dtype)
        w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(dtype)
        xd = x.to(cuda_device)
        out = ops.add_rmsnorm(xd, w.to(cuda_device), 1e-6, delta.to(cuda_device))
        x_ref = x + delta
        xf = x_ref.float()
        ref = w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(dtype)
        assert torch.equal(xd.cpu(), x_ref)
        assert torch.allclose(out.cpu().float(), ref.float(), rtol=2 ** -7, atol=1e-3)
        assert (out.cpu() != ref).float().mean() < 0.01
        plain = ops.add_rmsnorm(x.to(cuda_device), w.to(cuda_device), 1e-6)
        xf = x.float()
        assert (plain.cpu() != w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(dtype)).float().mean() < 0.01
    ops.check_status(cuda_device)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("k_before_rotation", [False, True])
def test_rope_and_page_write_in_one_launch(ops, cuda_device, dtype, k_before_rotation):
    """`rope_store` = `rope_inplace` on the q and k heads + `store_kvcache_unified_layout` of k and v, bit for bit: rotated rows in
    the buffer, rotated (or, on request, un-rotated) k and v rows at their slots, untouched pages elsewhere, skipped negative
    slots, a reported out-of-range slot; without a slot mapping only the rotation happens."""
    g = torch.Generator().manual_seed(123)
    t, hq, hkv, d, pages, page = 45, 4, 2, 128, 3, 32
    buf = torch.randn(t, (hq + 2 * hkv) * d + 64, generator=g).to(dtype)          # a padded row stride
    pos = torch.randint(0, 30000, (t,), generator=g)
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2).float() / d))
    emb = torch.cat((pos.float().unsqueeze(-1) * inv,) * 2, dim=-1)
    cos, sin = emb.cos().to(dtype).to(cuda_device), emb.sin().to(dtype).to(cuda_device)
    slots = torch.randperm(pages * page, generator=g)[:t].to(torch.int32)
    slots[5] = -1
    kc0 = torch.randn(pages, page, hkv, d, generator=g).to(dtype)
    vc0 = torch.randn(pages, page, hkv, d, generator=g).to(dtype)

    def view(b):
        return b[:, : (hq + 2 * hkv) * d].view(t, hq + 2 * hkv, d)

    ref_buf, ref_k, ref_v = buf.to(cuda_device), kc0.to(cuda_device), vc0.to(cuda_device)
    rq = view(ref_buf)
    if k_before_rotation:
        ops.store_kvcache_unified_layout(rq[:, hq:hq + hkv], rq[:, hq + hkv:], ref_k, ref_v, slots.to(cuda_device), "diffusion_lm")
    ops.rope_inplace(rq[:, : hq + hkv], cos, sin)
    if not k_before_rotation:
        ops.store_kvcache_unified_layout(rq[:, hq:hq + hkv], rq[:, hq + hkv:], ref_k, ref_v, slots.to(cuda_device), "diffusion_lm")
    got_buf, got_k, got_v = buf.to(cuda_device), kc0.to(cuda_device), vc0.to(cuda_device)
    ops.rope_store(view(got_buf), cos, sin, hq, hkv, got_k, got_v, slots.to(cuda_device), k_before_rotation=k_before_rotation)
    ops.check_status(cuda_device)
    assert torch.equal(got_buf, ref_buf) and torch.equal(got_k, ref_k) and torch.equal(got_v, ref_v)
    only = buf.to(cuda_device)
    ops.rope_store(view(only), cos, sin, hq, hkv)
    assert torch.equal(only, ref_buf)
    bad = slots.clone()
    bad[0] = pages * page
    ops.rope_store(view(buf.to(cuda_device)), cos, sin, hq, hkv, got_k, got_v, bad.to(cuda_device))
    with pytest.raises(RuntimeError):
        ops.check_status(cuda_device)
    with pytest.raises(NotImplementedError):
        ops.rope_store(view(buf.float().to(cuda_device)), cos.float(), sin.float(), hq, hkv)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_dense_row_ops_match_eager(ops, cuda_device, dtype):
    """RMSNorm (+ residual add), in-place RoPE on a strided QKV buffer and SiLU*mul against the eager expressions of the
    model they replace, with eager's rounding of every intermediate (bit-exact in bf16 except where a reduction order
    can move the last bit of the fp32 mean)."""
    g = torch.Generator().manual_seed(90)
    t, hidden, hq, hkv, d, inter = 37, 512, 4, 2, 128, 688
    x = torch.randn(t, hidden, generator=g).to(dtype)
    delta = torch.randn(t, hidden, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(dtype)
    xd, dd = x.to(cuda_device), delta.to(cuda_device)
    out = ops.add_rmsnorm(xd, w.to(cuda_device), 1e-6, dd)
    x_ref = x + delta
    xf = x_ref.float()
    ref = w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(dtype)
    assert torch.equal(xd.cpu(), x_ref)
    tol = dict(rtol=1e-5, atol=1e-6) if dtype == torch.float32 else dict(rtol=2 ** -7, atol=1e-3)
    assert torch.allclose(out.cpu().float(), ref.float(), **tol)
    if dtype == torch.bfloat16:   # all but a stray last-bit difference are identical (fp32: the reduction order shows)
        assert (out.cpu() != ref).float().mean() < 0.01
    plain = ops.add_rmsnorm(x.to(cuda_device), w.to(cuda_device), 1e-6)
    xf = x.float()
    assert torch.allclose(plain.cpu().float(), (w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(dtype)).float(), **tol)
    # rope on the q and k heads of a fused [T, hq + 2 hkv, d] buffer; v must stay untouched
    qkv = torch.randn(t, hq + 2 * hkv, d, generator=g).to(dtype)
    pos = torch.randint(0, 30000, (t,), generator=g)
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2).float() / d))
    emb = torch.cat((pos.float().unsqueeze(-1) * inv,) * 2, dim=-1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    dev = qkv.to(cuda_device)
    ops.rope_inplace(dev[:, : hq + hkv], cos.to(cuda_device), sin.to(cuda_device))
    part = qkv[:, : hq + hkv]
    rot = torch.cat((-part[..., d // 2:], part[..., : d // 2]), dim=-1)
    assert torch.equal(dev.cpu()[:, : hq + hkv], part * cos.unsqueeze(1) + rot * sin.unsqueeze(1))
    assert torch.equal(dev.cpu()[:, hq + hkv:], qkv[:, hq + hkv:])
    gu = torch.randn(t, 2 * inter, generator=g).to(dtype)
    got = ops.silu_mul(gu.to(cuda_device)).cpu()
    want = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
    assert torch.allclose(got.float(), want.float(), **tol)
    if dtype == torch.bfloat16:
        assert (got != want).float().mean() < 0.01


# ----------------------------------------------------------------------------------------------- linear layers
def _linear_reference(x, w, bias, silu):
    """fp32 on the CPU from the same bf16 / fp16 operands, rounded as the unfused sequence rounds."""
    acc = x.float() @ w.float().t()
    if bias is not None:
        acc = acc + bias.float()
    if not silu:
        return acc
    y = acc.to(x.dtype).float()
    gate, up = y[:, 0::2], y[:, 1::2]
    return (torch.nn.functional.silu(gate).to(x.dtype).float() * up)


def _assert_within_one_ulp(out, ref32, dtype):
    """The kernel accumulates in fp32 and rounds once: its result is the rounded reference up to one unit in the last place
    (different summation order), never more. Outputs that cancel to nearly zero are measured against a floor of 5 % of the
    mean magnitude: there the fp32 summation error of the terms, not the final rounding, sets the difference."""
    out = out.float().cpu()
    ulp = torch.finfo(dtype).eps * ref32.abs().clamp_min(0.05 * float(ref32.abs().mean()))
    worst = float(((out - ref32).abs() / ulp).max())
    assert worst <= 1.01, f"{worst:.2f} ulp"
    exact = float((out == ref32.to(dtype).float()).float().mean())
    assert exact > 0.97, exact


@pytest.mark.parametrize("m", [1, 4, 32, 33, 96, 128])
def test_linear_few_rows_streams_the_weights(ops, cuda_device, m):
    """M <= 128: weights on the 128-row side of the instruction, k-blocks dealt over all SMs (stream-K), shares of a feature
    tile summed through the workspace. Shapes include a K that is not a multiple of 64 and an N that is not a multiple of
    128; the second call reuses the workspace (the arrival counters must have returned to zero)."""
    g = torch.Generator().manual_seed(60 + m)
    for (n, k, with_bias) in ((1024, 512, True), (2752, 1376, False), (4608, 3584, True), (300, 512, False)):
        x = (torch.randn(m, k, generator=g) * 0.5).bfloat16()
        w = (torch.randn(n, k, generator=g) * 0.05).bfloat16()
        b = torch.randn(n, generator=g).bfloat16() if with_bias else None
        ref = _linear_reference(x, w, b, False)
        xd, wd, bd = x.to(cuda_device), w.to(cuda_device), None if b is None else b.to(cuda_device)
        out = ops.linear(xd, wd, bd)
        again = ops.linear(xd, wd, bd)
        ops.check_status(cuda_device)
        _assert_within_one_ulp(out, ref, torch.bfloat16)
        assert torch.equal(out, again), (m, n, k)


@pytest.mark.parametrize("m", [129, 549, 1200])
def test_linear_many_rows(ops, cuda_device, m):
    """M > 128: token tiles on the 128-row side, 256- or 128-wide feature tiles, ragged last tiles in M, N and K; fp16 too."""
    g = torch.Generator().manual_seed(70 + m)
    for (n, k, with_bias, dtype) in ((1024, 512, True, torch.bfloat16), (2752, 1376, False, torch.bfloat16), (4096, 512, False, torch.float16),
                                     (37888, 512, False, torch.bfloat16)):
        x = (torch.randn(m, k, generator=g) * 0.5).to(dtype)
        w = (torch.randn(n, k, generator=g) * 0.05).to(dtype)
        b = torch.randn(n, generator=g).to(dtype) if with_bias else None
        out = ops.linear(x.to(cuda_device), w.to(cuda_device), None if b is None else b.to(cuda_device))
        ops.check_status(cuda_device)
        _assert_within_one_ulp(out, _linear_reference(x, w, b, False), dtype)


@pytest.mark.parametrize("m", [32, 100, 700])
def test_linear_fused_silu_mul(ops, cuda_device, m):
    """Gate and up rows interleaved in the weight, SiLU(gate)·up in the epilogue: equal to projection -> silu_mul kernel."""
    g = torch.Generator().manual_seed(80 + m)
    inter, k = 1376, 512
    x = (torch.randn(m, k, generator=g) * 0.5).bfloat16().to(cuda_device)
    gate = (torch.randn(inter, k, generator=g) * 0.1).bfloat16().to(cuda_device)
    up = (torch.randn(inter, k, generator=g) * 0.1).bfloat16().to(cuda_device)
    fused = ops.linear(x, torch.stack([gate, up], dim=1).reshape(2 * inter, k).contiguous(), silu_mul_interleaved=True)
    unfused = ops.silu_mul(ops.linear(x, torch.cat([gate, up], dim=0).contiguous()))
    ops.check_status(cuda_device)
    assert fused.shape == (m, inter)
    if m > 128:
        assert torch.equal(fused, unfused)      # same k order per feature: the same bits
    else:
        # stream-K cuts a feature's k range at other points when its row moves to another tile: last-bit differences only
        diff = (fused.float() - unfused.float()).abs()
        assert float((diff > 0).float().mean()) < 0.02
        assert float((diff / (torch.finfo(torch.bfloat16).eps * unfused.float().abs().clamp_min(1e-3))).max()) <= 2.01
    ref = _linear_reference(x.cpu(), torch.stack([gate, up], dim=1).reshape(2 * inter, k).cpu(), None, True)
    assert rel_err(fused, ref) < 5e-3


def test_linear_cta_pairs(ops, cuda_device):
    """512 rows and more with at least one 256-wide feature tile per SM: 256 x 256 tiles worked by pairs of CTAs (one MMA over two
    SMs, each CTA staging its token rows and half of the weight rows). Ragged last tiles in M (a second CTA with no rows at
    all), N and K, bias, fp16, and the fused activation; every tile is whole, so the fused result has the unfused one's bits."""
    g = torch.Generator().manual_seed(91)
    for (m, n, k, with_bias, dtype) in ((1300, 4000, 1376, True, torch.bfloat16), (513, 37888, 512, False, torch.float16),
                                        (2049, 5120, 704, True, torch.bfloat16), (640, 9472, 256, False, torch.bfloat16),
                                        (1300, 4096, 4160, True, torch.bfloat16)):     # its last wave is cut along K, two pairs per tile
        x = (torch.randn(m, k, generator=g) * 0.5).to(dtype)
        w = (torch.randn(n, k, generator=g) * 0.05).to(dtype)
        b = torch.randn(n, generator=g).to(dtype) if with_bias else None
        xd, wd, bd = x.to(cuda_device), w.to(cuda_device), None if b is None else b.to(cuda_device)
        out = ops.linear(xd, wd, bd)
        again = ops.linear(xd, wd, bd)
        ops.check_status(cuda_device)
        _assert_within_one_ulp(out, _linear_reference(x, w, b, False), dtype)
        assert torch.equal(out, again), (m, n, k)
    m, inter, k = 1300, 4096, 512
    x = (torch.randn(m, k, generator=g) * 0.5).bfloat16().to(cuda_device)
    gate = (torch.randn(inter, k, generator=g) * 0.1).bfloat16().to(cuda_device)
    up = (torch.randn(inter, k, generator=g) * 0.1).bfloat16().to(cuda_device)
    fused = ops.linear(x, torch.stack([gate, up], dim=1).reshape(2 * inter, k).contiguous(), silu_mul_interleaved=True)
    unfused = ops.silu_mul(ops.linear(x, torch.cat([gate, up], dim=0).contiguous()))
    ops.check_status(cuda_device)
    assert torch.equal(fused, unfused)


def test_linear_rejects_what_it_cannot_run(ops, cuda_device):
    x = torch.zeros(8, 64, dtype=torch.float32, device=cuda_device)
    with pytest.raises(NotImplementedError):
        ops.linear(x, torch.zeros(16, 64, dtype=torch.float32, device=cuda_device))          # fp32: not a tensor-core dtype here
    xb = torch.zeros(8, 60, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(NotImplementedError):
        ops.linear(xb, torch.zeros(16, 60, dtype=torch.bfloat16, device=cuda_device))         # K not a multiple of 8
    assert ops.linear(torch.zeros(0, 64, dtype=torch.bfloat16, device=cuda_device), torch.zeros(16, 64, dtype=torch.bfloat16, device=cuda_device)).shape == (0, 16)
