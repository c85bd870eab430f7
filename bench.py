#!/usr/bin/env python3
"""Benchmark of the hot path: op-level non-contiguous paged decode attention.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
        bench.py --gpus N --steps K --warmup W

One step = one attention pass over one batch: 8 requests per GPU, each with 64 query + 32 response rows attending
4 selected chunks (16 pages of 256 tokens, any physical order, no gather) plus the bidirectional new rows;
28 query / 4 KV heads, head_dim 128, bf16. Decode is data-parallel over requests, so every rank runs its own batch
(weak scaling, no data-path collective). Prints ONE JSON line on rank 0.

Timing: CUDA events on the launching stream, max over ranks. Consecutive steps use different block tables that
together cover the whole 537 MB pool, so a step never finds its pages in the 126 MB L2.
`--impl reference` times the CPU restatement of the reference's own path (oracle/, all host threads) on a bounded
sample of the same workload; it is the only place the product bench executes the oracle, and only as the thing
being compared against.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

# ---- workload: BASELINE.json configs[1] ------------------------------------------------------------------
NUM_REQ = 8
HQ, HKV, D = 28, 4, 128
PAGE = 256
CHUNKS_IN_POOL, CHUNK_TOKENS, SEL_CHUNKS = 32, 1024, 4
QUERY_ROWS, RESP_ROWS = 64, 32
ROWS = QUERY_ROWS + RESP_ROWS
PAGES_PER_CHUNK = CHUNK_TOKENS // PAGE
CTX = SEL_CHUNKS * CHUNK_TOKENS
N_TABLES = CHUNKS_IN_POOL // SEL_CHUNKS  # disjoint selections that together touch the whole pool

FLOPS_PER_STEP = NUM_REQ * 4 * HQ * D * ROWS * (CTX + ROWS)                        # QK^T and PV
BYTES_PER_STEP = NUM_REQ * (CTX * 2 * HKV * D * 2 + ROWS * (2 * HQ + 2 * HKV) * D * 2)  # KV pages + q/k/v/out rows
# dram__bytes_read.sum + dram__bytes_write.sum of one attn_sm100_kernel launch on this workload, from the ncu capture
# summarised in profiles/attn_sm100_kernel_op_config.md (algorithmic minimum: BYTES_PER_STEP)
TRAFFIC_BYTES_PER_LAUNCH = 79_097_088
WORKLOAD = ("configs[1] op-level paged decode attention: 8 req x (64 query + 32 response rows), 28/4 heads, d128, "
            "page 256, 4 of 32 chunks (4096 ctx tokens) per request via block table, bidirectional, N(0,1) bf16")


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as handle:
            data = json.load(handle)
        return dict(hbm=float(data["hbm_gbs"]), tflops=float(data["bf16_tflops"]), source="measured")
    return dict(hbm=6650.0, tflops=1590.0, source="fallback")


class ClockSampler:
    """Samples SM clock and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._pump, daemon=True)
        self.thread.start()

    def _pump(self):
        for line in self.proc.stdout:
            self.samples.append(line.strip())

    def stop(self):
        if self.proc is None:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["nvidia-smi unavailable"])
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, sm_max, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.samples:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 6:
                continue
            try:
                sm.append(float(parts[0]))
                sm_max = float(parts[1])
            except ValueError:
                continue
            for name, val in zip(names, parts[2:6]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        sm.sort()
        return dict(sm_mhz=sm[len(sm) // 2] if sm else None, sm_max_mhz=sm_max, reasons=sorted(reasons), samples=len(sm))


def build_batch(seed: int, device: torch.device):
    """Seeded synthetic batch of the op-level config. The pool is N(0,1) bf16; block tables come from seeded
    permutations; N_TABLES tables per request pick disjoint chunk sets so that rotating them sweeps the pool."""
    g = torch.Generator().manual_seed(seed)
    pages_per_req = CHUNKS_IN_POOL * PAGES_PER_CHUNK
    num_pages = NUM_REQ * pages_per_req
    k_cache = torch.randn(num_pages, PAGE, HKV, D, generator=g, dtype=torch.float32).to(torch.bfloat16)
    v_cache = torch.randn(num_pages, PAGE, HKV, D, generator=g, dtype=torch.float32).to(torch.bfloat16)
    tables = torch.empty(N_TABLES, NUM_REQ, SEL_CHUNKS * PAGES_PER_CHUNK, dtype=torch.int32)
    for r in range(NUM_REQ):
        perm = torch.randperm(CHUNKS_IN_POOL, generator=g)
        for t in range(N_TABLES):
            chosen = perm[t * SEL_CHUNKS:(t + 1) * SEL_CHUNKS].tolist()
            ids = [r * pages_per_req + c * PAGES_PER_CHUNK + i for c in chosen for i in range(PAGES_PER_CHUNK)]
            tables[t, r] = torch.tensor(ids, dtype=torch.int32)
    total = NUM_REQ * ROWS
    q = torch.randn(total, HQ, D, generator=g).to(torch.bfloat16)
    k = torch.randn(total, HKV, D, generator=g).to(torch.bfloat16)
    v = torch.randn(total, HKV, D, generator=g).to(torch.bfloat16)
    cu = torch.arange(0, total + 1, ROWS, dtype=torch.int32)
    seq_lens = torch.full((NUM_REQ,), CTX + ROWS, dtype=torch.int32)
    host = dict(q=q, k=k, v=v, k_cache=k_cache, v_cache=v_cache, tables=tables, cu=cu, seq_lens=seq_lens)
    if device.type == "cpu":
        return host, None
    dev = {name: t.to(device) for name, t in host.items()}
    return host, dev


def run_native(args, rank: int, world: int, local_rank: int):
    from prefilling_dllm_b200 import ops

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    host, dev = build_batch(1000 + rank, device)
    out = torch.empty_like(dev["q"])
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream(device)

    def step(i: int):
        ops.paged_attention(dev["q"], dev["k"], dev["v"], out, cu_seqlens_q=dev["cu"], max_query_len=ROWS,
                            key_cache=dev["k_cache"], value_cache=dev["v_cache"], block_table=dev["tables"][i % N_TABLES],
                            seq_lens=dev["seq_lens"], max_seq_len=CTX + ROWS, sm_scale=scale, bidirectional=True)

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize(device)
    ops.check_status(device)
    # launches per step: the attention kernel (split-KV partials are merged inside it by the last CTA of a tile pair;
    # the 4-byte-per-pair arrival counters are cleared by a memset node, not a kernel)
    launches_per_step = 1

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    sampler = ClockSampler(local_rank)
    if rank == 0:
        sampler.start()

    # ---- device-resident timing (value) ----
    barrier()
    torch.cuda.synchronize(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(args.steps):
        step(i)
    stop.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    ms_total = start.elapsed_time(stop)

    # ---- end to end through the reference-facing op with HOST buffers (e2e) ----
    # Every step copies its q/k/v rows and block table from pinned host memory, runs the op, and copies the output back to
    # pinned host memory. The three stages run on three streams over three sets of device buffers, so step i's download,
    # step i+1's kernel and step i+2's upload overlap (PCIe is full duplex); all of it is inside the timed region.
    # host rows in the fused [T, Hq + 2 Hkv, D] layout a QKV projection produces: one upload per step; the op takes q, k, v
    # as strided views of it
    pin_qkv = torch.cat([host["q"], host["k"], host["v"]], dim=1).contiguous().pin_memory()
    tables_pin = host["tables"].pin_memory()
    n_buf = 3
    bufs = []
    for _ in range(n_buf):
        qkv = torch.empty(pin_qkv.shape, dtype=pin_qkv.dtype, device=device)
        bufs.append(dict(qkv=qkv, q=qkv[:, :HQ], k=qkv[:, HQ:HQ + HKV], v=qkv[:, HQ + HKV:],
                         table=torch.empty_like(dev["tables"][0]), out=torch.empty_like(dev["q"]),
                         out_host=torch.empty_like(host["q"]).pin_memory(),
                         up=torch.cuda.Event(), done=torch.cuda.Event(), down=torch.cuda.Event()))
    s_up, s_run, s_down = torch.cuda.Stream(device), torch.cuda.Stream(device), torch.cuda.Stream(device)
    h2d = pin_qkv.numel() * 2 + bufs[0]["table"].numel() * 4
    d2h = bufs[0]["out_host"].numel() * 2
    e2e_steps = args.steps

    def e2e_step(i: int):
        b = bufs[i % n_buf]
        torch.cuda.set_stream(s_up)
        s_up.wait_event(b["down"])            # the buffers' previous output has left the device
        b["qkv"].copy_(pin_qkv, non_blocking=True)
        b["table"].copy_(tables_pin[i % N_TABLES], non_blocking=True)
        b["up"].record(s_up)
        torch.cuda.set_stream(s_run)
        s_run.wait_event(b["up"])
        ops.diffusion_lm_parallel_flash_decoding(b["q"], b["k"], b["v"], b["out"], "auto", dev["k_cache"], dev["v_cache"], b["table"],
                                                 dev["cu"], dev["seq_lens"], CTX + ROWS, ROWS, 1.0, 1.0, RESP_ROWS, None, None, scale,
                                                 None, True)
        b["done"].record(s_run)
        torch.cuda.set_stream(s_down)
        s_down.wait_event(b["done"])
        b["out_host"].copy_(b["out"], non_blocking=True)
        b["down"].record(s_down)
        torch.cuda.set_stream(stream)

    def join():
        for st in (s_up, s_run, s_down):
            stream.wait_stream(st)

    for st in (s_up, s_run, s_down):
        st.wait_stream(stream)
    for b in bufs:
        b["down"].record(s_down)
    for i in range(3):
        e2e_step(i)
    join()
    torch.cuda.synchronize(device)
    barrier()
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for st in (s_up, s_run, s_down):
        st.wait_stream(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    join()
    e_stop.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms_total = e_start.elapsed_time(e_stop)
    # the last step's output, read on the host, must be the kernel's: compare with the device-resident result of the same table
    step((e2e_steps - 1) % N_TABLES)
    torch.cuda.synchronize(device)
    if not torch.equal(bufs[(e2e_steps - 1) % n_buf]["out_host"], out.cpu()):
        raise RuntimeError("end-to-end output differs from the device-resident run of the same inputs")
    clocks = sampler.stop() if rank == 0 else None
    ops.check_status(device)

    if world > 1:
        t = torch.tensor([ms_total, e2e_ms_total], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_total, e2e_ms_total = float(t[0]), float(t[1])
    if rank != 0:
        return None

    ms_per_step = ms_total / args.steps
    tokens_per_step = world * NUM_REQ * ROWS
    value = tokens_per_step / (ms_per_step * 1e-3)
    e2e_value = tokens_per_step / (e2e_ms_total / e2e_steps * 1e-3)
    peaks = load_peaks()
    achieved_tf = FLOPS_PER_STEP / (ms_per_step * 1e-3) / 1e12
    achieved_gb = BYTES_PER_STEP / (ms_per_step * 1e-3) / 1e9
    traffic = TRAFFIC_BYTES_PER_LAUNCH
    line = {
        "metric": "decode_attention_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "requests_per_gpu": NUM_REQ, "rows_per_request": ROWS, "ctx_tokens": CTX,
                   "parallelism": f"dp{world} (replicas over requests, no data-path collective)",
                   "l2": f"{N_TABLES} disjoint block tables rotate over a 537 MB K/V pool (> 126 MB L2) between steps"},
        "roofline": {"bound": "tensor", "achieved": achieved_tf, "peak": peaks["tflops"], "unit": "TFLOP/s",
                     "frac": achieved_tf / peaks["tflops"], "traffic": traffic, "peak_source": peaks["source"] + " (burst bf16 GEMM)",
                     "flops_per_launch": FLOPS_PER_STEP, "hbm": {"achieved": achieved_gb, "peak": peaks["hbm"], "unit": "GB/s",
                                                                "frac": achieved_gb / peaks["hbm"], "bytes_per_launch": BYTES_PER_STEP}},
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms_total / e2e_steps},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    if world == 1:
        line["cpu_baseline"] = cpu_baseline(sample_requests=2)
    return line


def cpu_baseline(sample_requests: int, repeats: int = 1):
    """The CPU restatement of the reference path, timed on the host cores over a bounded sample of the batch."""
    from oracle import hotpath as oracle

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    host, _ = build_batch(1000, torch.device("cpu"))
    rows = sample_requests * ROWS
    args = dict(cu_seqlens_q=host["cu"][: sample_requests + 1].tolist(), k_cache=host["k_cache"], v_cache=host["v_cache"],
                block_table=host["tables"][0][:sample_requests], seq_lens=host["seq_lens"][:sample_requests].tolist(),
                sm_scale=1.0 / math.sqrt(D), bidirectional=True)
    warm = dict(args, cu_seqlens_q=[0, ROWS], block_table=host["tables"][0][:1], seq_lens=[CTX + ROWS])
    oracle.paged_attention(host["q"][:ROWS], host["k"][:ROWS], host["v"][:ROWS], **warm)  # warm-up: one request
    t0 = time.perf_counter()
    for _ in range(repeats):
        oracle.paged_attention(host["q"][:rows], host["k"][:rows], host["v"][:rows], **args)
    dt = (time.perf_counter() - t0) / repeats
    return {"value": rows / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{sample_requests} of the batch's {NUM_REQ} requests ({rows} rows), fp32 torch on CPU, {dt:.2f} s"}


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return None
    steps = max(1, args.steps)
    warm = max(0, args.warmup)
    # every step is the same bounded sample; keep the whole run within a few minutes
    per = 1
    for _ in range(min(warm, 1)):
        cpu_baseline(sample_requests=per)
    t0 = time.perf_counter()
    results = [cpu_baseline(sample_requests=per) for _ in range(min(steps, 5))]
    wall = time.perf_counter() - t0
    value = sum(r["value"] for r in results) / len(results)
    base = results[-1]
    base["value"] = value
    return {
        "impl": "reference", "metric": "decode_attention_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": len(results), "warmup": min(warm, 1), "ms_per_step": wall / len(results) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": base["sample"]},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_request(args, rank: int, world: int, local_rank: int):
    """End-to-end request latency and decode rate of the whole hot path at BASELINE configs[2] / configs[3] shapes:
    Dream-7B architecture (random init, bf16), random prefix + 64-token query through the eval-class runtime.

    dream7b_8k : 8192-token prefix, chunk 1024, top-4, joint full_prompt_mask prefill, 32 new tokens, ONE GPU per replica
                 (with --gpus N every rank serves its own request: weak scaling, no collective).
    dream7b_32k: 32768-token prefix, 32 chunks, top-8, token_capacity 256, chunk_query mode, 64 new tokens; chunk scoring
                 and chunk prefill sharded over the N ranks (score all-gather, KV hand-off to the decode rank)."""
    from prefilling_dllm_b200 import ops
    from prefilling_dllm_b200.model import DreamArch, PagedDreamModel
    from prefilling_dllm_b200.parallelcomp import FastDLLMParallelComp, FastDLLMParallelCompConfig
    from prefilling_dllm_b200.sharded import ShardedChunkPrefill

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    long_ctx = args.workload == "dream7b_32k"
    prefix_len, topk, new_tokens = (32768, 8, 64) if long_ctx else (8192, 4, 32)
    model = PagedDreamModel.random_init(DreamArch.dream_7b(), device=device, dtype=torch.bfloat16, num_pages=160, page_size=256, seed=0)
    cfg = FastDLLMParallelCompConfig(
        fastdllm_dream_dir="", pretrained="", device="cuda", dtype="bfloat16", chunk_size=1024, topk_chunks=topk,
        score_mode="draft_self_information", score_draft_tokens=4, score_draft_partial_rounds=1, score_context_mode="single_chunk",
        score_attention_mask="causal", score_batch_size=8, block_length=32, max_new_tokens=new_tokens, threshold=0.9, temperature=0.0,
        cache_build_mode="chunk_query" if long_ctx else "full_prompt_mask",
        chunk_position_mode="reuse" if long_ctx else "continuous",
        query_position_mode="after_reused_window" if long_ctx else "after_selected_chunks",
        token_capacity=256 if long_ctx else 0)
    rt = FastDLLMParallelComp(cfg, model=model)
    sharded = ShardedChunkPrefill(rt) if (long_ctx and world > 1) else None
    gen = torch.Generator().manual_seed(0 if long_ctx else rank)
    context = torch.randint(0, 151000, (prefix_len,), generator=gen).tolist()
    query = torch.randint(0, 151000, (64,), generator=gen).tolist()

    def request():
        if sharded is not None:
            return sharded.generate(prefix_ids=rt.bos_ids(), context_ids=context, query_ids=query, decode_rank=0)
        return rt.generate(prefix_ids=rt.bos_ids(), context_ids=context, query_ids=query)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)

    steps, warmup = max(1, min(args.steps, 20)), max(3, min(args.warmup, 5))
    for _ in range(warmup):
        request()
    ops.check_status(device)
    sampler = ClockSampler(local_rank)
    if rank == 0:
        sampler.start()
    decode_s0 = rt.total_generation_time
    phase = {"decode": 0.0}
    inner = rt._denoise_blocks

    def timed_denoise(*a, **k):
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        out = inner(*a, **k)
        torch.cuda.synchronize(device)
        phase["decode"] += time.perf_counter() - t0
        return out

    rt._denoise_blocks = timed_denoise
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        request()
    stop.record()
    barrier()
    ms = torch.tensor([start.elapsed_time(stop) / steps], device=device)
    dec = torch.tensor([phase["decode"] / steps], device=device)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(dec, op=torch.distributed.ReduceOp.MAX)
    clocks = sampler.stop() if rank == 0 else None
    ops.check_status(device)
    if rank != 0:
        return None
    ms_per_request, decode_s = float(ms.item()), float(dec.item())
    requests_in_flight = 1 if long_ctx else world
    naive = None
    if args.naive and world == 1:
        # What the path avoids (the comparison the reference's README quotes): no selection, no cache — every denoise
        # step re-encodes [BOS ‖ context ‖ query ‖ generated ‖ block] bidirectionally on the same model and kernels; the LM
        # head runs on the block's 32 (shifted) rows only. One request, CUDA-event timed.
        mask_id = rt._mask_token_id()
        prompt = list(rt.bos_ids()) + context + query
        torch.cuda.synchronize(device)
        n_start, n_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_start.record()
        done, n_steps = [], 0
        with torch.inference_mode():
            while len(done) < new_tokens:
                blen = min(32, new_tokens - len(done))
                block = torch.full((blen,), mask_id, dtype=torch.int64, device=device)
                base = len(prompt) + len(done)
                while bool((block == mask_id).any()):
                    ids = torch.cat([rt.model.ids_tensor(prompt + done), block])
                    rows = list(range(base - 1, base + blen - 1))
                    logits, _ = rt._forward_packed([[0] * (base + blen)], [list(range(base + blen))], causal=False, ids_tensor=ids,
                                                   logit_rows=rows)
                    ops.unmask_step(logits, block, mask_token_id=mask_id, threshold=0.9, shift=False)
                    n_steps += 1
                done += block.tolist()
        n_stop.record()
        torch.cuda.synchronize(device)
        ops.check_status(device)
        naive_ms = n_start.elapsed_time(n_stop)
        naive = {"ms_per_request": naive_ms, "denoise_steps": n_steps, "rows_per_step": len(prompt) + new_tokens,
                 "speedup_of_this_path": naive_ms / ms_per_request}
    return {
        "metric": "request_latency_ms", "value": ms_per_request, "unit": "ms", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": ms_per_request, "higher_is_better": False, "scaling": "strong" if long_ctx else "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.workload}: Dream-7B architecture, random init, {prefix_len}-token random prefix + 64-token query, "
                               f"chunk 1024, top-{topk}, block 32, {new_tokens} new tokens, threshold 0.9, greedy, "
                               + ("token_capacity 256, chunk_query, chunks sharded over the ranks" if long_ctx else "full_prompt_mask"),
                   "parallelism": (f"chunks over {world} ranks, decode on rank 0" if long_ctx else f"dp{world} (one request per rank)")},
        "decode_tok_per_s": requests_in_flight * new_tokens / decode_s if decode_s > 0 else None,
        "decode_ms_per_request": decode_s * 1e3,
        "requests_per_s": requests_in_flight * 1e3 / ms_per_request,
        "full_reencode_every_step": naive,
        "clocks": clocks,
    }


def run_decode_batch(args, rank: int, world: int, local_rank: int):
    """Decode throughput of the PD engine facade with `--concurrent` requests per GPU sharing every denoise step:
    Dream-7B architecture (random init, bf16), each request a 4193-token prompt (what is left of an 8K prefix after
    top-4 chunk selection, plus the query) prefilled into pages beforehand; timed: `decode_from_pd_records` of one
    32-token block per request. Replicas over GPUs (every rank its own requests, no collective)."""
    from prefilling_dllm_b200 import ops
    from prefilling_dllm_b200.engine import FastDLLMDreamEngine
    from prefilling_dllm_b200.model import DreamArch, PagedDreamModel

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    # llada8b_decode_batch: the decode side of BASELINE configs[4] — LLaDA-8B architecture (32 MHA heads, un-shifted logits),
    # each request 4 selected chunks of 2048 tokens + a 64-token query in pages
    llada = args.workload == "llada8b_decode_batch"
    arch = DreamArch.llada_8b() if llada else DreamArch.dream_7b()
    name = "LLaDA-8B" if llada else "Dream-7B"
    n_req, prompt_len, block = max(1, args.concurrent), (4 * 2048 + 64 if llada else 4193), 32
    pages_per_req = -(-prompt_len // 256) + 1
    model = PagedDreamModel.random_init(arch, device=device, dtype=torch.bfloat16, num_pages=n_req * pages_per_req + 8, page_size=256)
    engine = FastDLLMDreamEngine(model, max_model_len=16384, block_length=block, mask_token_id=arch.mask_token_id, threshold=0.9,
                                 enforce_eager=False)
    gen = torch.Generator().manual_seed(100 + rank)
    prompts = [torch.randint(0, 126000, (prompt_len,), generator=gen).tolist() for _ in range(n_req)]

    def one_round():
        records = [engine.prefill_to_pd_record(p, max_new_tokens=block) for p in prompts]     # prefix-cache hits after the first round
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        outs = engine.decode_from_pd_records(records, max_new_tokens=block)
        torch.cuda.synchronize(device)
        return time.perf_counter() - t0, outs

    steps, warmup = max(1, min(args.steps, 10)), max(3, min(args.warmup, 4))
    for _ in range(warmup):
        one_round()
    ops.check_status(device)
    sampler = ClockSampler(local_rank)
    if rank == 0:
        sampler.start()
    if world > 1:
        torch.distributed.barrier()
    total, n_steps = 0.0, 0
    for _ in range(steps):
        dt, outs = one_round()
        total += dt
        n_steps = max(o.n_diff_steps for o in outs)
    sec = torch.tensor([total / steps], device=device)
    if world > 1:
        torch.distributed.all_reduce(sec, op=torch.distributed.ReduceOp.MAX)
    clocks = sampler.stop() if rank == 0 else None
    ops.check_status(device)
    if rank != 0:
        return None
    seconds = float(sec.item())
    return {
        "metric": "decode_tok_per_s", "value": world * n_req * block / seconds, "unit": "tok/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": seconds * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"{args.workload}: {n_req} concurrent requests per GPU, {name} architecture random init, {prompt_len}-token "
                               f"prompt in pages, one {block}-token block each, threshold 0.9, greedy; {n_steps} shared denoise steps per block",
                   "parallelism": f"dp{world} (replicas over requests, no data-path collective)"},
        "ms_per_denoise_step": seconds * 1e3 / max(1, n_steps), "clocks": clocks,
    }


def run_mha_decode_attention(args, rank: int, world: int, local_rank: int):
    """The HBM-bound side of the decode-attention kernel: LLaDA-8B-shaped heads (32 query = 32 KV heads, d128, bf16),
    `--concurrent` requests per GPU (default 16), each one 32-row response block attending 8256 cached tokens (4 selected
    chunks of 2048 + a 64-token query) through a block table of pages in random physical order. One attention launch
    per step = one layer of one denoise step. The K/V pool (2 x 1.1 GB at 16 requests) is far larger than L2.
    Replicas over GPUs (every rank its own requests, no collective)."""
    from prefilling_dllm_b200 import ops

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    n_req, rows, ctx, heads, page = max(1, args.concurrent), 32, 4 * 2048 + 64, 32, 256
    pages_per = -(-ctx // page)
    g = torch.Generator(device=device).manual_seed(2000 + rank)
    k_cache = torch.randn(n_req * pages_per, page, heads, D, device=device, dtype=torch.bfloat16, generator=g)
    v_cache = torch.randn(n_req * pages_per, page, heads, D, device=device, dtype=torch.bfloat16, generator=g)
    table = torch.randperm(n_req * pages_per, device=device, generator=g).to(torch.int32).view(n_req, pages_per).contiguous()
    qkv = torch.randn(n_req * rows, 3 * heads, D, device=device, dtype=torch.bfloat16, generator=g)
    q, k, v = qkv[:, :heads], qkv[:, heads:2 * heads], qkv[:, 2 * heads:]
    out = torch.empty(n_req * rows, heads, D, device=device, dtype=torch.bfloat16)
    cu = (torch.arange(n_req + 1, device=device) * rows).to(torch.int32)
    seq_lens = torch.full((n_req,), ctx + rows, dtype=torch.int32, device=device)
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream(device)

    def step():
        return ops.paged_attention(q, k, v, out, cu_seqlens_q=cu, max_query_len=rows, key_cache=k_cache, value_cache=v_cache,
                                   block_table=table, seq_lens=seq_lens, max_seq_len=pages_per * page + rows, sm_scale=scale,
                                   bidirectional=True)

    warmup = max(3, args.warmup)
    for _ in range(warmup):
        used = step()
    torch.cuda.synchronize(device)
    ops.check_status(device)
    if used != "tc":
        raise RuntimeError(f"expected the tcgen05 attention kernel, ran {used}")
    sampler = ClockSampler(local_rank)
    if rank == 0:
        sampler.start()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    stop.record(stream)
    torch.cuda.synchronize(device)
    ms = torch.tensor([start.elapsed_time(stop) / args.steps], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    clocks = sampler.stop() if rank == 0 else None
    ops.check_status(device)
    if rank != 0:
        return None
    ms_per_step = float(ms.item())
    bytes_per_launch = n_req * (ctx * 2 * heads * D * 2 + rows * 4 * heads * D * 2)     # K/V pages once + q, k, v, out rows
    flops_per_launch = n_req * 4 * heads * D * rows * (ctx + rows)
    peaks = load_peaks()
    gbs = bytes_per_launch / (ms_per_step * 1e-3) / 1e9
    return {
        "metric": "decode_attention_tok_per_s", "value": world * n_req * rows / (ms_per_step * 1e-3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"op_mha_decode: {n_req} req x 32 response rows, 32/32 heads (LLaDA-8B shape), d128, page 256, {ctx} cached "
                               "tokens per request via block table (random page order), bidirectional, N(0,1) bf16",
                   "parallelism": f"dp{world} (replicas over requests, no data-path collective)",
                   "l2": "K/V pool of 2 x %.2f GB read once per step (> 126 MB L2)" % (k_cache.numel() * 2 / 1e9)},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm"], "unit": "GB/s", "frac": gbs / peaks["hbm"],
                     # dram bytes of one launch at 16 requests from the ncu capture summarised in
                     # profiles/attn_sm100_kernel_mha_decode.md; other request counts were not captured
                     "traffic": 2_208_000_000 if n_req == 16 else None,
                     "peak_source": peaks["source"], "bytes_per_launch": bytes_per_launch,
                     "tensor": {"achieved": flops_per_launch / (ms_per_step * 1e-3) / 1e12, "unit": "TFLOP/s"}},
        "gpu_launches": args.steps, "clocks": clocks,
    }


def run_byte_kernels(args, local_rank: int):
    """Achieved HBM rate of each byte-moving kernel of the path at the shapes of BASELINE's Dream-7B configs, one GPU.
    Every kernel runs over several independent input sets in turn, together larger than L2 (so no launch finds its input
    in the 126 MB L2), as a replayed CUDA graph of 16 launches, CUDA-event timed; bytes are the algorithmic ones (inputs read once + outputs written once)."""
    from prefilling_dllm_b200 import ops

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(7)
    peaks = load_peaks()
    vocab, hkv, d, page = 152064, 4, D, PAGE
    results = []

    def timed(name, unit_note, nbytes, make_call, n_sets):
        # warm up eagerly (workspaces get allocated), then capture a graph of `calls` launches over the rotating input
        # sets and replay it: Python's per-call overhead (10-20 us) would otherwise hide kernels this short
        for i in range(max(3, args.warmup)):
            make_call(i % n_sets)
        torch.cuda.synchronize(device)
        calls = n_sets * max(1, 16 // n_sets)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=device)):
            for i in range(calls):
                make_call(i % n_sets)
        replays = max(3, min(args.steps, 200) // calls)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize(device)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(replays):
            graph.replay()
        stop.record()
        torch.cuda.synchronize(device)
        ops.check_status(device)
        us = start.elapsed_time(stop) / (replays * calls) * 1e3
        gbs = nbytes / us / 1e3
        results.append({"kernel": name, "shape": unit_note, "us": round(us, 2), "bytes": nbytes, "GB/s": round(gbs, 1),
                        "frac_of_hbm_peak": round(gbs / peaks["hbm"], 3)})

    # (4) unmask step: 16 requests x 32 rows of bf16 logits over the Dream vocabulary (one launch per request block,
    # as the engine issues them); 8 sets of 16 x 9.7 MB
    rows = 32
    logit_sets = [torch.randn(16, rows, vocab, device=device, dtype=torch.bfloat16, generator=g) for _ in range(2)]
    ids = torch.full((rows,), vocab - 1, dtype=torch.int64, device=device)
    last = torch.randn(vocab, device=device, dtype=torch.bfloat16, generator=g)

    ids_init = ids.clone()
    ids_init[0] = 5

    def unmask(i):
        ids.copy_(ids_init)
        ops.unmask_step(logit_sets[i % 2][i % 16], ids, mask_token_id=vocab - 1, threshold=0.9, last_logit=last, shift=True,
                        softmax_dtype=torch.float32)
    timed("unmask_kernel (+ a 256-byte copy that resets the block)", "[32, 152064] bf16 logits, one block", rows * vocab * 2, unmask, 32)

    # (2a) self-information tail: 8 chunks x 66 label rows of bf16 logits
    n_chunks, n_lab = 8, 66
    label_sets = [torch.randn(n_chunks * n_lab, vocab, device=device, dtype=torch.bfloat16, generator=g) for _ in range(2)]
    labels = torch.randint(0, vocab, (n_lab,), device=device, generator=g)
    timed("self_info_nll_kernel", "[8 x 66, 152064] bf16 label rows", n_chunks * n_lab * vocab * 2,
          lambda i: ops.self_information_scores(label_sets[i % 2], labels, n_chunks), 2)
    del logit_sets, label_sets

    # (5) KV page write: the 4193 rows of the joint prefill of one layer, K and V, read + write
    n_tok = 4193
    pool_pages = 640                                   # 2 x 335 MB per pool: rotating 16 disjoint slot sets sweeps it
    k_cache = torch.zeros(pool_pages, page, hkv, d, device=device, dtype=torch.bfloat16)
    v_cache = torch.zeros_like(k_cache)
    kv_sets = [torch.randn(n_tok, 2 * hkv, d, device=device, dtype=torch.bfloat16, generator=g) for _ in range(16)]
    slot_sets = [(torch.randperm(40 * page, device=device, generator=g)[:n_tok] + i * 40 * page).to(torch.int32) for i in range(16)]
    timed("store_unified_vec16_kernel", "4193 rows x (K + V) x 4 heads x 128, scattered slots", n_tok * 2 * hkv * d * 2 * 2,
          lambda i: ops.store_kvcache_unified_layout(kv_sets[i][:, :hkv], kv_sets[i][:, hkv:], k_cache, v_cache, slot_sets[i], "diffusion_lm"), 16)

    # PD snapshot / load of one layer plane: gather and scatter of 4161 prompt rows
    page_sets = [torch.randperm(pool_pages, device=device, generator=g)[:17].to(torch.int32) for _ in range(16)]
    n_rows = 4161
    timed("page_copy_kernel (gather)", "4161 rows x 4 heads x 128 out of 17 pages", n_rows * hkv * d * 2 * 2,
          lambda i: ops.gather_pages(k_cache, page_sets[i], n_rows), 16)
    dense = torch.randn(n_rows, hkv, d, device=device, dtype=torch.bfloat16, generator=g)
    timed("page_copy_kernel (scatter)", "4161 rows x 4 heads x 128 into 17 pages", n_rows * hkv * d * 2 * 2,
          lambda i: ops.scatter_pages(dense, k_cache, page_sets[i]), 16)

    # (2c) eviction scorer of one (chunk, layer): 8 window rows against prefix + chunk + window keys, 28/4 heads
    length, c_len, w = 1 + 1024 + 8, 1024, 8
    qk_sets = [(torch.randn(length, HQ, d, device=device, dtype=torch.bfloat16, generator=g),
                torch.randn(length, hkv, d, device=device, dtype=torch.bfloat16, generator=g)) for _ in range(8)]
    ev_bytes = length * hkv * d * 2 + w * HQ * d * 2 + HQ * c_len * 4
    timed("evict_logits + evict_reduce kernels", "L = 1033 keys, 8 query rows, 28/4 heads -> [28, 1024] fp32", ev_bytes,
          lambda i: ops.query_to_chunk_attention_scores(qk_sets[i][0], qk_sets[i][1], prefix_len=1, chunk_len=c_len, query_len=w,
                                                        scale=d ** -0.5, reduce_mode="sum", attention_mask="causal"), 8)
    head_scores = torch.rand(28, HQ, c_len, device=device, generator=g)
    timed("evict_select kernel (pool, reduce, rank)", "[28 layers, 28 heads, 1024] fp32 -> 256 kept per (layer, KV head)",
          head_scores.numel() * 4 + 28 * hkv * 256 * 8,
          lambda i: ops.evict_select(head_scores, num_kv_heads=hkv, keep_count=256, per_head=True), 1)
    return {
        "metric": "achieved_hbm_gb_per_s", "value": None, "unit": "GB/s", "n_gpus": 1, "steps": max(20, min(args.steps, 200)),
        "warmup": max(3, args.warmup), "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "byte_kernels: each HBM-bound kernel of the path at Dream-7B shapes, inputs rotated so that no launch "
                               "finds them in L2 (except evict_select, whose 3.2 MB input is L2-resident by design)"},
        "hbm_peak": peaks["hbm"], "peak_source": peaks["source"], "kernels": results,
    }


def run_step_breakdown(args, local_rank: int):
    """Where one denoise step of Dream-7B (32 block rows against 4161 cached tokens, bf16) spends its time: each group
    of launches captured in a CUDA graph of its own and replayed, CUDA-event timed. One GPU."""
    import torch.nn.functional as F

    from prefilling_dllm_b200 import ops
    from prefilling_dllm_b200.model import DreamArch, PagedDreamModel

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    arch = DreamArch.dream_7b()
    m = PagedDreamModel.random_init(arch, device=device, dtype=torch.bfloat16, num_pages=64, page_size=256)
    rows, ctx = 32, 4161
    hq, hkv, d, hidden, inter = arch.num_attention_heads, arch.num_key_value_heads, arch.head_dim, arch.hidden_size, arch.intermediate_size
    h = torch.randn(rows, hidden, device=device, dtype=torch.bfloat16)
    hi = torch.randn(rows, inter, device=device, dtype=torch.bfloat16)
    gu = torch.randn(rows, 2 * inter, device=device, dtype=torch.bfloat16)
    qkv = torch.randn(rows, hq + 2 * hkv, d, device=device, dtype=torch.bfloat16)
    cos, sin = m._rope_tables(torch.arange(rows, device=device) + ctx)
    n_pages = -(-ctx // 256)
    table = torch.arange(4 * -(-n_pages // 4), dtype=torch.int32, device=device).view(1, -1)
    seq_lens = torch.tensor([ctx + rows], dtype=torch.int32, device=device)
    cu = torch.tensor([0, rows], dtype=torch.int32, device=device)
    out = torch.empty(rows, hq, d, device=device, dtype=torch.bfloat16)
    kc, vc = m.layer_cache(0)
    layers = arch.num_hidden_layers

    def gemms():
        for w in m.layers:
            F.linear(h, w["wqkv"], w["bqkv"]); F.linear(h, w["wo"]); F.linear(h, w["wgu"]); F.linear(hi, w["wd"])
        F.linear(h, m.lm_head)

    def row_ops():
        for _ in range(layers):
            ops.add_rmsnorm(h, m.layers[0]["ln1"], 1e-6, h)
            ops.rope_inplace(qkv[:, : hq + hkv], cos.reshape(-1, d), sin.reshape(-1, d))
            ops.add_rmsnorm(h, m.layers[0]["ln2"], 1e-6, h)
            ops.silu_mul(gu)

    def attention():
        for _ in range(layers):
            ops.paged_attention(qkv[:, :hq], qkv[:, hq:hq + hkv], qkv[:, hq + hkv:], out, cu_seqlens_q=cu, max_query_len=rows, key_cache=kc,
                                value_cache=vc, block_table=table, seq_lens=seq_lens, max_seq_len=table.shape[1] * 256 + rows, sm_scale=d ** -0.5)

    def timed(fn):
        fn()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=device)):
            fn()
        for _ in range(3):
            graph.replay()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(max(5, min(args.steps, 20))):
            graph.replay()
        stop.record()
        torch.cuda.synchronize(device)
        return start.elapsed_time(stop) / max(5, min(args.steps, 20))

    t_gemm, t_rows, t_attn = timed(gemms), timed(row_ops), timed(attention)
    ops.check_status(device)
    weight_bytes = (sum(w[k].numel() for w in m.layers for k in ("wqkv", "wo", "wgu", "wd")) + m.lm_head.numel()) * 2
    kv_bytes = layers * (ctx * 2 * hkv * d * 2 + rows * (2 * hq + 2 * hkv) * d * 2)
    peaks = load_peaks()
    return {
        "metric": "denoise_step_ms", "value": t_gemm + t_rows + t_attn, "unit": "ms", "n_gpus": 1, "higher_is_better": False,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "dream7b_step: one denoise step of Dream-7B, 32 block rows, 4161 cached tokens, groups replayed as CUDA graphs"},
        "breakdown_ms": {"cublas_gemms": t_gemm, "row_ops_4_per_layer": t_rows, "attention_28_layers": t_attn},
        "gemm_weight_gbs": weight_bytes / (t_gemm * 1e-3) / 1e9, "attention_kv_gbs": kv_bytes / (t_attn * 1e-3) / 1e9,
        "hbm_peak_gbs": peaks["hbm"], "peak_source": peaks["source"],
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--workload", default="op", choices=["op", "op_mha_decode", "byte_kernels", "dream7b_8k", "dream7b_32k", "dream7b_step", "dream7b_decode_batch",
                             "llada8b_decode_batch"],
                    help="op (default): BASELINE configs[1], the op-level decode attention; op_mha_decode: the same kernel on an HBM-bound "
                         "MHA shape; the others time whole requests")
    ap.add_argument("--naive", action="store_true", help="dream7b_8k / dream7b_32k on one GPU: also time one request that "
                    "re-encodes the full context at every denoise step")
    ap.add_argument("--concurrent", type=int, default=16, help="requests per GPU that share a denoise step (dream7b_decode_batch)")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device: the product path has no CPU fallback")
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "op":
            line = run_native(args, rank, world, local_rank)
        elif args.workload == "op_mha_decode":
            line = run_mha_decode_attention(args, rank, world, local_rank)
        elif args.workload == "byte_kernels":
            line = run_byte_kernels(args, local_rank) if rank == 0 else None
        elif args.workload in ("dream7b_decode_batch", "llada8b_decode_batch"):
            line = run_decode_batch(args, rank, world, local_rank)
        elif args.workload == "dream7b_step":
            line = run_step_breakdown(args, local_rank) if rank == 0 else None
        else:
            line = run_request(args, rank, world, local_rank)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
