"""Host logic of the chunk-sharded prefill, on CPU with world_size-2 gloo ranks: ownership plan, the score all-gather,
the shared deterministic ranking, and the grouped point-to-point KV hand-off to the decode rank."""

import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from prefilling_dllm_b200.sharded import (ChunkShardPlan, all_gather_chunk_scores, exchange_chunk_kv, plan_kv_transfers, prefill_ranks,  # noqa: E402
                                          rank_chunks)


def test_plan_partitions_every_chunk_once():
    for n in (0, 1, 7, 8, 32, 33):
        for w in (1, 2, 3, 8):
            plan = ChunkShardPlan(n, w)
            owned = [c for r in range(w) for c in plan.chunks_of(r)]
            assert owned == list(range(n))
            assert all(plan.owner(c) == r for r in range(w) for c in plan.chunks_of(r))
            sizes = [len(plan.chunks_of(r)) for r in range(w)]
            assert max(sizes) - min(sizes) <= 1 and max(sizes, default=0) == plan.max_per_rank
    assert ChunkShardPlan(32, 8).chunks_of(3) == [12, 13, 14, 15]      # 4 chunks per GPU at 32 chunks on 8 GPUs
    with pytest.raises(IndexError):
        ChunkShardPlan(4, 2).owner(4)


def test_ranking_is_the_stable_descending_sort():
    assert rank_chunks([0.1, 0.5, 0.5, -1.0, 0.5], 2) == [1, 2]                   # ties: lower index first
    assert rank_chunks([0.1, 0.5, 0.5, -1.0, 0.5], 2, keep_first_chunk=True) == [0, 1, 2]
    assert rank_chunks([float("nan"), float("-inf"), -3.0], 1) == [2]
    assert rank_chunks([1.0, 2.0], 0) == [0, 1] and rank_chunks([], 4) == []


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_chunks, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = ChunkShardPlan(n_chunks, world)
        truth = torch.linspace(-3.0, 1.0, n_chunks).roll(3)          # every rank can recompute the expected result
        mine = plan.chunks_of(rank)
        scores = all_gather_chunk_scores(truth[mine].clone(), plan, rank)
        assert torch.equal(scores, truth)
        selected = rank_chunks(scores.tolist(), 3)
        kept = {ci: 4 + ci for ci in selected}
        shape = lambda k: (2, 2, k, 2, 8)  # noqa: E731
        payloads = {ci: torch.full(shape(kept[ci]), float(ci)) for ci in selected if plan.owner(ci) == rank}
        positions = {ci: torch.arange(kept[ci]) + 100 * ci for ci in selected if plan.owner(ci) == rank}
        transfers = plan_kv_transfers(selected, kept, plan)
        assert [t.order for t in transfers] == list(range(len(selected))) and [t.chunk_index for t in transfers] == selected
        decode_rank = world - 1
        got_kv, got_pos = exchange_chunk_kv(transfers, rank=rank, decode_rank=decode_rank, payloads=payloads, positions=positions,
                                            payload_shape=shape, dtype=torch.float32, device="cpu")
        if rank == decode_rank:
            assert sorted(got_kv) == selected
            for ci in selected:
                assert tuple(got_kv[ci].shape) == shape(kept[ci]) and bool((got_kv[ci] == float(ci)).all())
                assert got_pos[ci].tolist() == [100 * ci + i for i in range(kept[ci])]
        else:
            assert got_kv == {} and got_pos == {}
        # a payload that disagrees with the plan is refused before anything is posted
        if payloads:
            ci = next(iter(payloads))
            bad = dict(payloads)
            bad[ci] = bad[ci][:, :, :-1]
            if plan.owner(ci) != decode_rank:
                with pytest.raises(ValueError):
                    exchange_chunk_kv([t for t in transfers if t.chunk_index == ci], rank=rank, decode_rank=decode_rank, payloads=bad,
                                      positions=positions, payload_shape=shape, dtype=torch.float32, device="cpu")
        dist.barrier()
        out.put((rank, selected))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_chunks", [8, 7])
def test_two_ranks_agree_on_selection_and_hand_off_kv(n_chunks):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_chunks, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = dict(out.get(timeout=5) for _ in range(2))
    assert results[0] == results[1] and len(results[0]) == 3


def test_selected_chunks_are_dealt_evenly_for_the_prefill():
    """Selected chunks cluster (here six of eight in one rank's scoring range); their prefill is dealt round-robin from the
    decode rank, and the transfers follow that assignment."""
    selected = [8, 9, 10, 11, 12, 13, 20, 31]
    for world, decode_rank in ((2, 0), (4, 1), (8, 0), (3, 2)):
        ranks = prefill_ranks(selected, world, decode_rank)
        load = [sum(1 for r in ranks.values() if r == w) for w in range(world)]
        assert max(load) == -(-len(selected) // world) and ranks[selected[0]] == decode_rank
        plan = ChunkShardPlan(32, world)
        transfers = plan_kv_transfers(selected, {ci: 256 for ci in selected}, plan, ranks)
        assert [t.src_rank for t in transfers] == [ranks[ci] for ci in selected]
        assert [t.src_rank for t in plan_kv_transfers(selected, {ci: 256 for ci in selected}, plan)] == [plan.owner(ci) for ci in selected]
