#!/usr/bin/env python3
"""Benchmark of the Prefilling-dLLM long-context hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference] [--workload request|...]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
        bench.py --gpus N --steps K --warmup W

Default workload `request`. One step = ONE REQUEST through `FastDLLMParallelComp.generate`: Dream-7B architecture (28 layers,
hidden 3584, 28 / 4 heads of 128, MLP 18944, vocabulary 152064, random init, bf16), an 8192-token random prefix and a 64-token
query as host token-id lists in, 32 generated token ids as a host list out; chunk 1024 with chunk BOS, draft-self-information
scoring of the 8 chunks in one packed causal forward, top-4, one joint bidirectional prefill, confidence-threshold block
denoising (threshold 0.9, greedy). With N GPUs every rank serves its own request (decode is data-parallel over requests, no
data-path collective): weak scaling.

The ONE JSON line rank 0 prints:
  metric / value   decode tokens per second: generated tokens of all ranks / device time of the block-denoising phase (its
                   inputs, the KV pages, are resident in HBM when it starts), max over ranks
  ms_per_step      latency of one whole request, CUDA events, max over ranks
  e2e              tokens per second of the whole request (host ids in, host ids out), and that latency
  phases_ms        draft / scoring / prefill / decode split of one request (CUDA events at the phase boundaries)
  kernel_share     one denoise step by kernel group, each group replayed as a CUDA graph of its own
  roofline         the dominant kernel of the denoise step, the weight-streaming GEMM: algorithmic bytes / measured time
  ops              op-level measurements: the paged decode attention on the 8-request op shape and on MHA decode heads, the
                   attention kernel on the two prefill shapes of this request, the GEMM kernel next to cuBLAS
  request_32k      the 32768-token request (32 chunks, top-8, token_capacity 256, 64 new tokens) with chunk scoring and chunk
                   prefill SHARDED over the N ranks: score all-gather, kept-KV hand-off to the decode rank, bytes moved
  cpu_baseline     the reference's own class on the CPU toy, on this machine's host cores (N = 1 only), next to
  toy_same_config  this runtime on the same toy

`--impl reference` times that CPU run alone and prints it with "impl": "reference".
Consecutive requests differ in nothing but time: weights (15 GB) and KV pages are far larger than the 126 MB L2 and are
streamed again by every forward, so no step finds its inputs cached. LongBench-style data, checkpoints and tokenizers are
absent: inputs are seeded uniform random token ids of the same shapes.
"""

from __future__ import annotations

import argparse
import json
import gc
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

# ---- op-level workload: 8 requests x (64 query + 32 response rows) over 4 of 32 cached chunks -------------------------------
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
OP_WORKLOAD = ("op-level paged decode attention: 8 req x (64 query + 32 response rows), 28/4 heads, d128, "
               "page 256, 4 of 32 chunks (4096 ctx tokens) per request via block table, bidirectional, N(0,1) bf16")


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as handle:
            data = json.load(handle)
        return dict(hbm=float(data["hbm_gbs"]), tflops=float(data["bf16_tflops"]), tflops_sustained=float(data.get("bf16_tflops_sustained", data["bf16_tflops"])),
                    source="measured")
    return dict(hbm=6650.0, tflops=1590.0, tflops_sustained=1400.0, source="fallback")


def timed_launches(fn, n_sets: int, launches: int, device):
    """Average duration (us) of `fn(i)` over >= `launches` back-to-back launches, CUDA events on the current stream."""
    for i in range(max(3, n_sets)):
        fn(i)
    torch.cuda.synchronize(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(device)
    start.record(stream)
    for i in range(launches):
        fn(i)
    stop.record(stream)
    torch.cuda.synchronize(device)
    return start.elapsed_time(stop) / launches * 1e3


def timed_graph(fn, device, replays: int = 10):
    """ms of one execution of `fn()` replayed as a CUDA graph (no Python between its launches)."""
    fn()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=device)):
        fn()
    for _ in range(3):
        graph.replay()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(replays):
        graph.replay()
    stop.record()
    torch.cuda.synchronize(device)
    return start.elapsed_time(stop) / replays


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



def op_decode_attention(steps: int, warmup: int, rank: int, world: int, device: torch.device, *, with_e2e: bool = True):
    """The op-level decode attention shape: device-resident launches, and the reference-facing op with HOST buffers (every
    step copies q/k/v rows and the block table from pinned host memory and the output back, three streams over three
    buffer sets so that consecutive steps overlap on the full-duplex link). Returns a sub-record."""
    from prefilling_dllm_b200 import ops

    host, dev = build_batch(1000 + rank, device)
    out = torch.empty_like(dev["q"])
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream(device)
    steps = max(int(steps), 200)

    def step(i: int):
        ops.paged_attention(dev["q"], dev["k"], dev["v"], out, cu_seqlens_q=dev["cu"], max_query_len=ROWS,
                            key_cache=dev["k_cache"], value_cache=dev["v_cache"], block_table=dev["tables"][i % N_TABLES],
                            seq_lens=dev["seq_lens"], max_seq_len=CTX + ROWS, sm_scale=scale, bidirectional=True)

    us = timed_launches(step, N_TABLES, steps, device)
    ops.check_status(device)
    peaks = load_peaks()
    record = {
        "workload": OP_WORKLOAD, "launches": steps, "us_per_launch": us, "tok_per_s": NUM_REQ * ROWS / (us * 1e-6),
        "l2": f"{N_TABLES} disjoint block tables rotate over a 537 MB K/V pool (> 126 MB L2) between launches",
        "roofline": {"bound": "tensor", "achieved": FLOPS_PER_STEP / (us * 1e-6) / 1e12, "peak": peaks["tflops"], "unit": "TFLOP/s",
                     "frac": FLOPS_PER_STEP / (us * 1e-6) / 1e12 / peaks["tflops"], "traffic": TRAFFIC_BYTES_PER_LAUNCH,
                     "peak_source": peaks["source"] + " (burst bf16 GEMM)", "flops_per_launch": FLOPS_PER_STEP,
                     "hbm": {"achieved": BYTES_PER_STEP / (us * 1e-6) / 1e9, "peak": peaks["hbm"], "unit": "GB/s",
                             "frac": BYTES_PER_STEP / (us * 1e-6) / 1e9 / peaks["hbm"], "bytes_per_launch": BYTES_PER_STEP}},
    }
    if not with_e2e:
        return record
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
    e2e_steps = min(steps, 200)

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
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for st in (s_up, s_run, s_down):
        st.wait_stream(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    join()
    e_stop.record(stream)
    torch.cuda.synchronize(device)
    e2e_us = e_start.elapsed_time(e_stop) / e2e_steps * 1e3
    # the last step's output, read on the host, must be the kernel's: compare with the device-resident result of the same table
    step((e2e_steps - 1) % N_TABLES)
    torch.cuda.synchronize(device)
    if not torch.equal(bufs[(e2e_steps - 1) % n_buf]["out_host"], out.cpu()):
        raise RuntimeError("end-to-end output differs from the device-resident run of the same inputs")
    ops.check_status(device)
    record["host_buffers"] = {"us_per_step": e2e_us, "tok_per_s": NUM_REQ * ROWS / (e2e_us * 1e-6), "h2d_bytes_per_step": h2d,
                              "d2h_bytes_per_step": d2h}
    return record


def op_mha_decode(n_req: int, steps: int, rank: int, device: torch.device):
    """The HBM-bound side of the decode-attention kernel: LLaDA-8B-shaped heads (32 query = 32 KV heads, d128, bf16), `n_req`
    requests, each one 32-row block over 8256 cached tokens through a block table of pages in random physical order. One
    launch = one layer of one denoise step; the K/V pool (2 x 1.1 GB at 16 requests) is far larger than L2."""
    from prefilling_dllm_b200 import ops

    rows, ctx, heads, page = 32, 4 * 2048 + 64, 32, 256
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
    used = []

    def step(i):
        used.append(ops.paged_attention(q, k, v, out, cu_seqlens_q=cu, max_query_len=rows, key_cache=k_cache, value_cache=v_cache,
                                        block_table=table, seq_lens=seq_lens, max_seq_len=pages_per * page + rows, sm_scale=D ** -0.5,
                                        bidirectional=True))

    us = timed_launches(step, 1, max(50, min(steps, 200)), device)
    ops.check_status(device)
    if used[-1] != "tc":
        raise RuntimeError(f"expected the tcgen05 attention kernel, ran {used[-1]}")
    nbytes = n_req * (ctx * 2 * heads * D * 2 + rows * 4 * heads * D * 2)     # K/V pages once + q, k, v, out rows
    peaks = load_peaks()
    gbs = nbytes / us / 1e3
    return {"workload": f"{n_req} req x 32 response rows, 32/32 heads (LLaDA-8B shape), d128, page 256, {ctx} cached tokens per request "
                        "via block table (random page order), bidirectional, N(0,1) bf16",
            "us_per_launch": us, "tok_per_s": n_req * rows / (us * 1e-6),
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm"], "unit": "GB/s", "frac": gbs / peaks["hbm"],
                         # dram bytes of one launch at 16 requests, from the ncu capture in profiles/attn_sm100_kernel_mha_decode.md
                         "traffic": 2_208_000_000 if n_req == 16 else None, "peak_source": peaks["source"], "bytes_per_launch": nbytes}}


def op_decode_rows(device: torch.device, steps: int):
    """The attention launch of ONE request's denoise step: 32 block rows x 28 / 4 heads over 4161 cached tokens in 17 pages (random
    physical order) plus the block itself. HBM-bound in principle (8.8 MB of K/V, 1.3 us at the copy peak); in practice bound by
    the length of one CTA's dependent chain and the merge of the KV splits. Page sets rotate over a 335 MB pool (> L2)."""
    from prefilling_dllm_b200 import ops

    rows, ctx, pages_per, pool_pages = 32, 4161, 17, 640
    g = torch.Generator(device=device).manual_seed(5000)
    k_cache = torch.randn(pool_pages, PAGE, HKV, D, device=device, dtype=torch.bfloat16, generator=g)
    v_cache = torch.randn(pool_pages, PAGE, HKV, D, device=device, dtype=torch.bfloat16, generator=g)
    tables = torch.randperm(pool_pages, device=device, generator=g)[: 32 * pages_per].to(torch.int32).view(32, 1, pages_per)
    qkv = torch.randn(rows, HQ + 2 * HKV, D, device=device, dtype=torch.bfloat16, generator=g)
    out = torch.empty(rows, HQ, D, device=device, dtype=torch.bfloat16)
    cu = torch.tensor([0, rows], dtype=torch.int32, device=device)
    seq_lens = torch.tensor([ctx + rows], dtype=torch.int32, device=device)

    def step(i):
        ops.paged_attention(qkv[:, :HQ], qkv[:, HQ:HQ + HKV], qkv[:, HQ + HKV:], out, cu_seqlens_q=cu, max_query_len=rows, key_cache=k_cache,
                            value_cache=v_cache, block_table=tables[i % 32], seq_lens=seq_lens, max_seq_len=pages_per * PAGE + rows, sm_scale=D ** -0.5)

    step(0)
    used_clusters = bool(ops.LAST_ATTENTION_USED_CLUSTERS)
    us = timed_graph(lambda: [step(i) for i in range(32)], device, replays=max(3, min(steps, 10))) / 32 * 1e3
    ops.check_status(device)
    nbytes = ctx * 2 * HKV * D * 2 + rows * (2 * HQ + 2 * HKV) * D * 2
    peaks = load_peaks()
    return {"workload": "1 request x 32 block rows, 28/4 heads, d128, 4161 cached tokens in 17 pages + the block, bidirectional, bf16; launches replayed "
                        "as a CUDA graph of 32 over rotating page sets",
            "kernel": "attn_decode_sm100_kernel (KV splits of a unit = one thread-block cluster)" if used_clusters else "attn_sm100_kernel + attn_combine_kernel",
            "us_per_launch": us, "roofline": {"bound": "hbm", "achieved": nbytes / us / 1e3, "peak": peaks["hbm"], "unit": "GB/s",
                                              "frac": nbytes / us / 1e3 / peaks["hbm"], "bytes_per_launch": nbytes, "traffic": None}}


def op_prefill_attention(device: torch.device, steps: int):
    """The attention kernel on the two prefill shapes of the 8K request (28 / 4 heads, d128, bf16, no cached context):
    scoring = 8 packed causal rows of 1093 tokens; joint prefill = one bidirectional sequence of 4193 tokens. Tensor-bound:
    FLOPs = 4 Hq D x visible (row, key) pairs. Inputs (19 / 36 MB per launch incl. output) rotate over 8 sets (> L2)."""
    from prefilling_dllm_b200 import ops

    peaks = load_peaks()
    g = torch.Generator(device=device).manual_seed(3000)
    out_rec = {}
    for name, lens, causal in (("scoring_causal_8x1093", [1093] * 8, True), ("joint_bidirectional_4193", [4193], False)):
        total = sum(lens)
        sets = [torch.randn(total, HQ + 2 * HKV, D, device=device, dtype=torch.bfloat16, generator=g) for _ in range(8)]
        out = torch.empty(total, HQ, D, device=device, dtype=torch.bfloat16)
        cu = torch.tensor([0] + [sum(lens[:i + 1]) for i in range(len(lens))], dtype=torch.int32, device=device)
        used = []

        def step(i):
            qkv = sets[i % 8]
            used.append(ops.paged_attention(qkv[:, :HQ], qkv[:, HQ:HQ + HKV], qkv[:, HQ + HKV:], out, cu_seqlens_q=cu, max_query_len=max(lens),
                                            sm_scale=D ** -0.5, causal=causal, bidirectional=True))

        us = timed_launches(step, 8, max(20, min(steps, 100)), device)
        ops.check_status(device)
        pairs = sum(n * (n + 1) // 2 if causal else n * n for n in lens)
        flops = 4 * HQ * D * pairs
        nbytes = total * (2 * HQ + 2 * HKV) * D * 2
        tf = flops / us / 1e6
        out_rec[name] = {"kernel": used[-1], "us_per_launch": us, "flops_per_launch": flops, "bytes_per_launch": nbytes,
                         "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["tflops"], "unit": "TFLOP/s", "frac": tf / peaks["tflops"],
                                      "peak_source": peaks["source"] + " (burst bf16 GEMM)", "traffic": None}}
        del sets
    return out_rec


def op_linear(device: torch.device, steps: int, only: str = ""):
    """The GEMM kernel on the linear-layer shapes of the 8K request, next to cuBLAS (torch.matmul) on the same operands:
    32 block rows (weight streaming: GB/s of weight bytes against the HBM peak) and the 8744 scoring rows (TFLOP/s against the
    bf16 peak). Weights rotate over several copies (> L2); launches replayed as CUDA graphs of 8."""
    from prefilling_dllm_b200 import ops

    peaks = load_peaks()
    g = torch.Generator(device=device).manual_seed(4000)
    rec = {}
    shapes = [("qkv", 4608, 3584), ("o", 3584, 3584), ("gate_up", 37888, 3584), ("down", 3584, 18944), ("lm_head", 152064, 3584)]
    for m in (32, 512, 8744):          # one block of rows, 16 blocks sharing a step, the scoring prefill
        for name, n, k in shapes:
            if (m > 128 and name == "lm_head") or (only and only != f"{name}_m{m}"):
                continue
            copies = max(2, min(8, int(300e6 // (n * k * 2)) + 1))
            ws = [torch.randn(n, k, device=device, dtype=torch.bfloat16, generator=g) * 0.02 for _ in range(copies)]
            x = torch.randn(m, k, device=device, dtype=torch.bfloat16, generator=g)
            out = torch.empty(m, n, device=device, dtype=torch.bfloat16)
            calls = 8
            t_mine = timed_graph(lambda: [ops.linear(x, ws[i % copies], out=out, weights_at_rest=True) for i in range(calls)], device, replays=max(3, min(steps, 10))) / calls * 1e3
            t_lib = timed_graph(lambda: [torch.matmul(x, ws[i % copies].t(), out=out) for i in range(calls)], device, replays=max(3, min(steps, 10))) / calls * 1e3
            ops.check_status(device)
            nbytes = (n * k + m * k + m * n) * 2
            flops = 2 * m * n * k
            entry = {"m": m, "n": n, "k": k, "us": t_mine, "cublas_us": t_lib}
            if m <= 128:
                entry["roofline"] = {"bound": "hbm", "achieved": nbytes / t_mine / 1e3, "peak": peaks["hbm"], "unit": "GB/s",
                                     "frac": nbytes / t_mine / 1e3 / peaks["hbm"], "bytes_per_launch": nbytes}
            else:
                entry["roofline"] = {"bound": "tensor", "achieved": flops / t_mine / 1e6, "peak": peaks["tflops_sustained"], "unit": "TFLOP/s",
                                     "frac": flops / t_mine / 1e6 / peaks["tflops_sustained"], "flops_per_launch": flops,
                                     "peak_source": peaks["source"] + " (sustained bf16 GEMM: timed back to back)"}
            rec[f"{name}_m{m}"] = entry
            del ws
    return rec


def reference_triton_on_this_gpu(device: torch.device):
    """The reference's own Triton kernels (staged unmodified under oracle/_ref/ops by oracle/build_ref.py), timed on this GPU on
    the same inputs as the library's kernels: 5 warm-ups, 20 timed launches, CUDA events (the protocol of the reference's
    examples/bench_unified_vs_distinct.py). A same-box baseline; nothing of it runs in the product path."""
    from oracle import build_ref
    from prefilling_dllm_b200 import ops

    try:
        ref = build_ref.load_engine_ops()
    except Exception as exc:
        return {"unavailable": f"{type(exc).__name__}: {exc}"}
    rec = {"vllm_stand_in": bool(ref.stubbed_vllm)}
    host, dev = build_batch(1000, device)
    scale = 1.0 / math.sqrt(D)

    def timed(fn):
        for _ in range(5):
            fn()
        torch.cuda.synchronize(device)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(20):
            fn()
        stop.record()
        torch.cuda.synchronize(device)
        return start.elapsed_time(stop) / 20 * 1e3

    try:
        # decode attention on the op shape: the reference reads the vLLM-style distinct layout
        pages, page, hkv, d = dev["k_cache"].shape
        kd = dev["k_cache"].view(pages, page, hkv, d // 8, 8).permute(0, 2, 3, 1, 4).contiguous()
        vd = dev["v_cache"].permute(0, 2, 3, 1).contiguous()
        mask = torch.ones(ROWS, ROWS, dtype=torch.bool, device=device)
        out_ref, out_mine = torch.empty_like(dev["q"]), torch.empty_like(dev["q"])
        table = dev["tables"][0]
        us_ref = timed(lambda: ref.chunked_prefill_paged_decode(dev["q"], dev["k"], dev["v"], out_ref, "auto", kd, vd, table, dev["cu"], dev["seq_lens"],
                                                                CTX + ROWS, ROWS, 1.0, 1.0, diffusion_blk_sz=32, sm_scale=scale, mask=mask, bidirectional=True))
        us_mine = timed(lambda: ops.diffusion_lm_parallel_flash_decoding(dev["q"], dev["k"], dev["v"], out_mine, "auto", dev["k_cache"], dev["v_cache"], table,
                                                                         dev["cu"], dev["seq_lens"], CTX + ROWS, ROWS, 1.0, 1.0, 32, None, None, scale, None, True))
        err = float((out_mine.float() - out_ref.float()).norm() / out_ref.float().norm())
        rec["decode_attention_op_shape"] = {"reference_triton_us": us_ref, "library_us": us_mine, "speedup": us_ref / us_mine, "rel_diff": err,
                                            "note": "one block table (pages stay L2-resident across the 20 launches of either side)"}
        del kd, vd
        # page write of 4193 rows (K and V)
        n_tok = 4193
        kv = torch.randn(n_tok, 2 * HKV, D, device=device, dtype=torch.bfloat16)
        slots = torch.randperm(pages * page, device=device)[:n_tok].to(torch.int32)
        kc, vc = torch.zeros_like(dev["k_cache"][:64]), torch.zeros_like(dev["v_cache"][:64])
        slots64 = (slots % (64 * page)).to(torch.int32)
        us_ref = timed(lambda: ref.store_kvcache_unified_layout(kv[:, :HKV], kv[:, HKV:], kc, vc, slots64, "diffusion_lm"))
        us_mine = timed(lambda: ops.store_kvcache_unified_layout(kv[:, :HKV], kv[:, HKV:], kc, vc, slots64, "diffusion_lm"))
        rec["page_write_4193_rows"] = {"reference_triton_us": us_ref, "library_us": us_mine, "speedup": us_ref / us_mine}
        # eviction scorer of one (chunk, layer)
        length = 1 + 1024 + 8
        q = torch.randn(length, HQ, D, device=device, dtype=torch.bfloat16)
        k = torch.randn(length, HKV, D, device=device, dtype=torch.bfloat16)
        kw = dict(prefix_len=1, chunk_len=1024, query_len=8, scale=scale, reduce_mode="sum", attention_mask="causal")
        us_ref = timed(lambda: ref.query_to_chunk_attention_scores(q, k, **kw))
        us_mine = timed(lambda: ops.query_to_chunk_attention_scores(q, k, **kw))
        rec["eviction_scorer_chunk_1024"] = {"reference_triton_us": us_ref, "library_us": us_mine, "speedup": us_ref / us_mine}
        ops.check_status(device)
    except Exception as exc:   # a reference kernel that does not run on this GPU / Triton version: record it, time nothing more
        rec["error"] = f"{type(exc).__name__}: {str(exc)[:300]}"
    return rec


# ---- whole requests ---------------------------------------------------------------------------------------------------------
README_FLAGS = dict(score_mode="draft_self_information", score_draft_tokens=4, score_draft_partial_rounds=1, score_context_mode="single_chunk",
                    score_attention_mask="causal", score_batch_size=8, block_length=32, threshold=0.9, temperature=0.0)


class PhaseTimer:
    """CUDA-event pairs around bound methods of a runtime: where one request spends its device time."""

    def __init__(self, device):
        self.device = device
        self.spans = []
        self.undo = []

    def wrap(self, obj, attr: str, name: str):
        inner = getattr(obj, attr)

        def timed(*a, **k):
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            try:
                return inner(*a, **k)
            finally:
                stop.record()
                self.spans.append((name, start, stop))

        setattr(obj, attr, timed)
        self.undo.append((obj, attr, inner))

    def restore(self):
        for obj, attr, inner in self.undo:
            setattr(obj, attr, inner)
        self.undo = []

    def totals_ms(self):
        torch.cuda.synchronize(self.device)
        out = {}
        for name, start, stop in self.spans:
            out[name] = out.get(name, 0.0) + start.elapsed_time(stop)
        self.spans = []
        return out


def denoise_step_breakdown(model, rows: int, ctx: int, device):
    """One denoise step of `rows` block rows over `ctx` cached tokens, by kernel group; every group is captured in a CUDA graph
    of its own with the model's real weights (15 GB, streamed from HBM by every replay) and timed by CUDA events."""
    from prefilling_dllm_b200 import ops

    a = model.arch
    hq, hkv, d, hidden, inter = a.num_attention_heads, a.num_key_value_heads, a.head_dim, a.hidden_size, a.intermediate_size
    dt = model.dtype
    h = torch.randn(rows, hidden, device=device, dtype=dt)
    hi = torch.randn(rows, inter, device=device, dtype=dt)
    attn = torch.randn(rows, hq * d, device=device, dtype=dt)
    qkv = torch.randn(rows, hq + 2 * hkv, d, device=device, dtype=dt)
    logits = torch.randn(1, rows, a.vocab_size, device=device, dtype=dt)
    block = torch.full((1, rows), a.mask_token_id, dtype=torch.int64, device=device)
    last = torch.randn(1, a.vocab_size, device=device, dtype=dt)
    cos, sin = model._rope_tables(torch.arange(rows, device=device) + ctx)
    n_pages = -(-ctx // model.page_size)
    table = torch.arange(4 * -(-n_pages // 4), dtype=torch.int32, device=device).view(1, -1) % model.num_pages
    seq_lens = torch.tensor([ctx + rows], dtype=torch.int32, device=device)
    cu = torch.tensor([0, rows], dtype=torch.int32, device=device)
    out = torch.empty(rows, hq, d, device=device, dtype=dt)
    slots = torch.full((rows,), -1, dtype=torch.int32, device=device)
    layers = a.num_hidden_layers

    def linears():
        for w in model.layers:
            ops.linear(h, w["wqkv"], w["bqkv"], weights_at_rest=True); ops.linear(attn, w["wo"], weights_at_rest=True)
            ops.linear(h, w["wgu"], silu_mul_interleaved=True, weights_at_rest=True); ops.linear(hi, w["wd"], weights_at_rest=True)
        ops.linear(h, model.lm_head, weights_at_rest=True)

    def row_ops():
        for li in range(layers):
            kc, vc = model.layer_cache(li)
            ops.add_rmsnorm(h, model.layers[li]["ln1"], a.rms_norm_eps, h)
            ops.rope_store(qkv, cos.reshape(-1, d), sin.reshape(-1, d), hq, hkv, kc, vc, slots)
            ops.add_rmsnorm(h, model.layers[li]["ln2"], a.rms_norm_eps, h)
        ops.add_rmsnorm(h, model.final_norm, a.rms_norm_eps)

    def attention():
        for li in range(layers):
            kc, vc = model.layer_cache(li)
            ops.paged_attention(qkv[:, :hq], qkv[:, hq:hq + hkv], qkv[:, hq + hkv:], out, cu_seqlens_q=cu, max_query_len=rows, key_cache=kc,
                                value_cache=vc, block_table=table, seq_lens=seq_lens, max_seq_len=table.shape[1] * model.page_size + rows,
                                sm_scale=d ** -0.5)

    def unmask():
        ops.unmask_step_batched(logits, block, mask_token_id=a.mask_token_id, threshold=0.9, last_logit=last, shift=a.logit_shift)

    t_lin, t_rows, t_attn, t_unm = (timed_graph(f, device) for f in (linears, row_ops, attention, unmask))
    ops.check_status(device)
    n_linear = 4 * layers + 1
    weight_bytes = (sum(w[k].numel() for w in model.layers for k in ("wqkv", "wo", "wgu", "wd")) + model.lm_head.numel()) * 2
    act_bytes = layers * rows * (hidden + (hq + 2 * hkv) * d + hq * d + hidden + hidden + inter + inter + hidden) * 2 + rows * (hidden + a.vocab_size) * 2
    kv_bytes = layers * (ctx * 2 * hkv * d * 2 + rows * (2 * hq + 2 * hkv) * d * 2)
    total = t_lin + t_rows + t_attn + t_unm
    return {
        "rows": rows, "cached_tokens": ctx, "sum_of_groups_ms": total,
        "groups_ms": {"linear_sm100_kernel": t_lin, "attention (+ split-KV merge)": t_attn, "rmsnorm / rope + page write": t_rows, "unmask_kernel": t_unm},
        "share": {"linear_sm100_kernel": t_lin / total, "attention": t_attn / total, "row_ops": t_rows / total, "unmask": t_unm / total},
        "launches": {"linear_sm100_kernel": n_linear, "attention": layers, "row_ops": 3 * layers + 1, "unmask": 1},
        "linear_bytes": weight_bytes + act_bytes, "linear_ms": t_lin, "linear_launches": n_linear,
        "attention_kv_gbs": kv_bytes / (t_attn * 1e-3) / 1e9,
    }


def build_dream7b(device):
    from prefilling_dllm_b200.model import DreamArch, PagedDreamModel

    return PagedDreamModel.random_init(DreamArch.dream_7b(), device=device, dtype=torch.bfloat16, num_pages=192, page_size=256, seed=0)


def make_runtime(model, *, long_ctx: bool):
    from prefilling_dllm_b200.parallelcomp import FastDLLMParallelComp, FastDLLMParallelCompConfig

    cfg = FastDLLMParallelCompConfig(
        fastdllm_dream_dir="", pretrained="", device="cuda", dtype="bfloat16", chunk_size=1024, topk_chunks=8 if long_ctx else 4,
        max_new_tokens=64 if long_ctx else 32,
        cache_build_mode="chunk_query" if long_ctx else "full_prompt_mask",
        chunk_position_mode="reuse" if long_ctx else "continuous",
        query_position_mode="after_reused_window" if long_ctx else "after_selected_chunks",
        token_capacity=256 if long_ctx else 0, **README_FLAGS)
    return FastDLLMParallelComp(cfg, model=model)


def timed_requests(request, steps: int, warmup: int, device, barrier):
    """(ms per request, result of the last one): CUDA events around `steps` back-to-back calls after `warmup` untimed ones."""
    for _ in range(warmup):
        request()
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    result = None
    for _ in range(steps):
        result = request()
    stop.record()
    barrier()
    return start.elapsed_time(stop) / steps, result


def run_request_once(local_rank: int):
    """ONE cold 8K request and nothing else: the command a profiler's launch list is taken from (every kernel of a request, a
    few ten thousand launches, no warm-up to skip)."""
    from prefilling_dllm_b200 import ops

    device = torch.device("cuda", local_rank)
    model = build_dream7b(device)
    rt = make_runtime(model, long_ctx=False)
    gen = torch.Generator().manual_seed(0)
    context = torch.randint(0, 151000, (8192,), generator=gen).tolist()
    query = torch.randint(0, 151000, (64,), generator=gen).tolist()
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    result = rt.generate(prefix_ids=rt.bos_ids(), context_ids=context, query_ids=query)
    torch.cuda.synchronize(device)
    ops.check_status(device)
    return {"workload": "one cold 8K request (Dream-7B architecture, random init)", "wall_ms": (time.perf_counter() - t0) * 1e3,
            "selected_chunks": list(result.selected_chunk_indices), "c_abi_calls": ops.C_ABI_CALLS}


def run_full_reencode(args, local_rank: int):
    """`--workload full_reencode --ctx 8192|32768`: what the path avoids, the comparison the reference's README quotes. No selection and
    no cache: every denoise step forwards [BOS, context, query, generated, block] bidirectionally on the same model and kernels, the
    LM head on the block's (shifted) rows only. One request, CUDA events, next to the same request through the path."""
    from prefilling_dllm_b200 import ops

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    long_ctx = args.ctx > 8192
    model = build_dream7b(device)
    rt = make_runtime(model, long_ctx=long_ctx)
    gen = torch.Generator().manual_seed(args.ctx)
    context = torch.randint(0, 151000, (args.ctx,), generator=gen).tolist()
    query = torch.randint(0, 151000, (64,), generator=gen).tolist()
    new_tokens = rt.max_new_tokens
    path_ms, _ = timed_requests(lambda: rt.generate(prefix_ids=rt.bos_ids(), context_ids=context, query_ids=query), max(1, min(args.steps, 3)),
                                max(3, args.warmup), device, lambda: torch.cuda.synchronize(device))
    mask_id = rt._mask_token_id()
    prompt = list(rt.bos_ids()) + context + query
    torch.cuda.synchronize(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    done, n_steps = [], 0
    with torch.inference_mode():
        while len(done) < new_tokens:
            blen = min(32, new_tokens - len(done))
            block = torch.full((blen,), mask_id, dtype=torch.int64, device=device)
            base = len(prompt) + len(done)
            while bool((block == mask_id).any()):
                ids = torch.cat([rt.model.ids_tensor(prompt + done), block])
                logits, _ = rt._forward_packed([[0] * (base + blen)], [list(range(base + blen))], causal=False, ids_tensor=ids,
                                               logit_rows=list(range(base - 1, base + blen - 1)))
                ops.unmask_step(logits, block, mask_token_id=mask_id, threshold=0.9, shift=False)
                n_steps += 1
            done += block.tolist()
    stop.record()
    torch.cuda.synchronize(device)
    ops.check_status(device)
    naive_ms = start.elapsed_time(stop)
    return {"metric": "request_latency_ms", "value": path_ms, "unit": "ms", "n_gpus": 1, "steps": 1, "warmup": max(3, args.warmup),
            "higher_is_better": False, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"Dream-7B architecture (random init), {args.ctx}-token random prefix + 64-token query, {new_tokens} new tokens, "
                                   "block 32, threshold 0.9: the path against re-encoding the full context at every denoise step"},
            "full_reencode_every_step": {"ms_per_request": naive_ms, "denoise_steps": n_steps, "rows_per_step": len(prompt) + new_tokens,
                                         "speedup_of_this_path": naive_ms / path_ms}}


def _write_random_dream7b_checkpoint(path: str, device, *, single_file: bool):
    """config.json, a stub tokenizer and bf16 N(0, 0.02) weights of the Dream-7B architecture under HF parameter names, for the
    reference's own loaders (its engine reads any *.safetensors; the eval-class plug-in contract reads one model.safetensors).
    Returns (mask_token_id, bos_token_id)."""
    import json as _json
    import shutil

    from safetensors.torch import save_file
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import Whitespace

    from oracle import build_ref

    hidden, inter, layers, hq, hkv, d, vocab, mask_id, bos = 3584, 18944, 28, 28, 4, 128, 152064, 151666, 151643
    cfg = dict(model_type="Dream", architectures=["DreamModel"], auto_map={"AutoConfig": "configuration_dream.DreamConfig"},
               vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_hidden_layers=layers, num_attention_heads=hq,
               num_key_value_heads=hkv, max_position_embeddings=131072, rope_theta=1000000.0, rms_norm_eps=1e-6, hidden_act="silu",
               mask_token_id=mask_id, pad_token_id=bos, bos_token_id=bos, eos_token_id=bos, torch_dtype="bfloat16", tie_word_embeddings=False)
    with open(os.path.join(path, "config.json"), "w") as handle:
        _json.dump(cfg, handle)
    if build_ref.engine_staged():
        shutil.copyfile(os.path.join(build_ref.REF_DIR, "engine", "configuration_dream.py"), os.path.join(path, "configuration_dream.py"))
    tok = Tokenizer(WordLevel({"<pad>": 0, "<bos>": 1, "<eos>": 2, "<mask>": 3}, unk_token="<pad>"))
    tok.pre_tokenizer = Whitespace()
    tok.save(os.path.join(path, "tokenizer.json"))
    with open(os.path.join(path, "tokenizer_config.json"), "w") as handle:
        _json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "bos_token": "<bos>", "eos_token": "<eos>", "mask_token": "<mask>",
                    "pad_token": "<pad>", "unk_token": "<pad>"}, handle)
    g = torch.Generator(device=device).manual_seed(0)

    def rnd(*shape):
        return (torch.randn(*shape, device=device, dtype=torch.float32, generator=g) * 0.02).to(torch.bfloat16).cpu()

    tensors = {"model.embed_tokens.weight": rnd(vocab, hidden), "lm_head.weight": rnd(vocab, hidden),
               "model.norm.weight": torch.ones(hidden, dtype=torch.bfloat16)}
    if not single_file:
        save_file(tensors, os.path.join(path, "model-head.safetensors"))
        tensors = {}
    for i in range(layers):
        p = f"model.layers.{i}."
        tensors.update({p + "self_attn.q_proj.weight": rnd(hq * d, hidden), p + "self_attn.q_proj.bias": rnd(hq * d),
                        p + "self_attn.k_proj.weight": rnd(hkv * d, hidden), p + "self_attn.k_proj.bias": rnd(hkv * d),
                        p + "self_attn.v_proj.weight": rnd(hkv * d, hidden), p + "self_attn.v_proj.bias": rnd(hkv * d),
                        p + "self_attn.o_proj.weight": rnd(hidden, hq * d), p + "mlp.gate_proj.weight": rnd(inter, hidden),
                        p + "mlp.up_proj.weight": rnd(inter, hidden), p + "mlp.down_proj.weight": rnd(hidden, inter),
                        p + "input_layernorm.weight": torch.ones(hidden, dtype=torch.bfloat16),
                        p + "post_attention_layernorm.weight": torch.ones(hidden, dtype=torch.bfloat16)})
        if not single_file:
            save_file(tensors, os.path.join(path, f"model-layer{i:02d}.safetensors"))
            tensors = {}
    if single_file:
        save_file(tensors, os.path.join(path, "model.safetensors"))
    return mask_id, bos


def run_reference_class_8k(args, local_rank: int):
    """`--workload reference_class_8k`: the UNMODIFIED reference eval class (`FastDLLMParallelComp`, staged under oracle/_ref/eval)
    with `device="cuda"` on THIS GPU on the 8K request of the default line, over the restated Dream plug-in model
    (oracle/contract_model: the Fast-dLLM v1 model the reference imports by directory is absent) with random-init Dream-7B
    weights in bf16. Phases timed by wrapping its bound methods between device synchronisations. A same-box baseline of the
    reference's host logic and cache handling on a plain PyTorch model; nothing of it runs in the product path."""
    import shutil
    import tempfile
    import traceback

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    out = {"metric": "decode_tok_per_s", "unit": "tok/s", "n_gpus": 1, "impl": "reference_class_same_gpu", "dtype": "bf16", "data": "synthetic",
           "higher_is_better": True, "steps": max(1, min(args.steps, 2)), "warmup": 1,
           "config": {"workload": "the reference's FastDLLMParallelComp (device=cuda) on this GPU over the restated Dream plug-in model: Dream-7B "
                                  "architecture (random init, bf16), 8192-token random prefix + 64-token query, chunk 1024 with chunk BOS, "
                                  "draft-self-information scoring at batch 8, top-4, joint full_prompt_mask prefill, block 32, 32 new tokens, threshold 0.9"}}
    tmp = tempfile.mkdtemp(prefix="pdllm_ref_class_")
    try:
        from oracle import build_ref

        ref = build_ref.load_eval_module()
        _write_random_dream7b_checkpoint(tmp, device, single_file=True)
        runtime = ref.load_fastdllm_parallelcomp(pretrained=tmp, fastdllm_dream_dir=os.path.join(ROOT, "oracle", "contract_model"), device=f"cuda:{local_rank}",
                                                 dtype="bfloat16", trust_remote_code=False, chunk_size=1024, topk_chunks=4, max_new_tokens=32,
                                                 max_length=16384, cache_build_mode="full_prompt_mask", chunk_position_mode="continuous",
                                                 query_position_mode="after_selected_chunks", token_capacity=0, **README_FLAGS)
        secs = {"draft": 0.0, "scoring": 0.0, "decode": 0.0}

        def timed(name, fn):
            def wrapper(*a, **k):
                torch.cuda.synchronize(device)
                t = time.perf_counter()
                try:
                    return fn(*a, **k)
                finally:
                    torch.cuda.synchronize(device)
                    secs[name] += time.perf_counter() - t
            return wrapper

        runtime._selection_query_ids_with_score_target = timed("draft", runtime._selection_query_ids_with_score_target)
        runtime.score_chunks_self_information_batched = timed("scoring", runtime.score_chunks_self_information_batched)
        runtime._denoise_block_confidence_threshold = timed("decode", runtime._denoise_block_confidence_threshold)
        gen = torch.Generator().manual_seed(0)
        context = torch.randint(0, 151000, (8192,), generator=gen).tolist()
        query = torch.randint(0, 151000, (64,), generator=gen).tolist()
        runs = []
        for it in range(out["steps"] + 1):
            for k in secs:
                secs[k] = 0.0
            torch.cuda.synchronize(device)
            t0 = time.perf_counter()
            result = runtime.generate(prefix_ids=runtime.bos_ids(), context_ids=context, query_ids=query)
            torch.cuda.synchronize(device)
            total = (time.perf_counter() - t0) * 1e3
            if it > 0:
                ph = {k: v * 1e3 for k, v in secs.items()}
                ph["prefill"] = max(0.0, total - sum(ph.values()))
                runs.append(dict(request_ms=total, phases_ms=ph, new_tokens=len(result.sequences), selected=list(result.selected_chunk_indices)))
        mean = {k: sum(r["phases_ms"][k] for r in runs) / len(runs) for k in ("draft", "scoring", "prefill", "decode")}
        total = sum(r["request_ms"] for r in runs) / len(runs)
        out.update(value=32 / (mean["decode"] * 1e-3), ms_per_step=total, phases_ms=mean, runs=runs,
                   e2e={"value": 32 / (total * 1e-3), "unit": "tok/s", "request_latency_ms": total})
    except BaseException as exc:
        out["unavailable"] = f"{type(exc).__name__}: {exc}"[:600]
        out["traceback"] = traceback.format_exc()[-3000:]
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return out


def run_reference_engine_8k(args, local_rank: int):
    """`--workload reference_engine_8k`: the UNMODIFIED reference PD engine (`FastDLLMDreamEngine`, staged under oracle/_ref/engine
    by oracle/build_ref.py) on THIS GPU on the 8K request of the default line: a random-init Dream-7B checkpoint is written to
    a temporary directory (bf16, the engine's deployment dtype), then draft + scoring of the 8 chunks
    (`select_chunks_by_engine`), the joint prefill of [BOS, 4 selected chunks, query] + 32 MASK slots (`prefill_to_pd_record`) and
    the block denoising (`decode_from_pd_record`) are timed with device synchronisation around each. A same-box baseline of the
    reference's own GPU code; nothing of it runs in the product path. If any step fails, the exception text is the result."""
    import json as _json
    import shutil
    import tempfile
    import traceback

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    out = {"metric": "decode_tok_per_s", "unit": "tok/s", "n_gpus": 1, "impl": "reference_engine_same_gpu", "dtype": "bf16", "data": "synthetic",
           "higher_is_better": True, "steps": max(1, min(args.steps, 2)), "warmup": 1,
           "config": {"workload": "the reference's FastDLLMDreamEngine on this GPU: Dream-7B architecture (random init, bf16), 8192-token random "
                                  "prefix in 8 chunks of 1024 (chunk BOS) + 64-token query, its own draft (4 tokens, 1 round) + per-chunk scoring, "
                                  "top-4, joint prefill, block 32, 32 new tokens, threshold 0.9, enforce_eager, flex attention backend"}}
    tmp = tempfile.mkdtemp(prefix="pdllm_ref_engine_")
    try:
        from oracle import build_ref

        module = build_ref.load_reference_engine()
        mask_id, bos = _write_random_dream7b_checkpoint(tmp, device, single_file=False)
        engine = module.FastDLLMDreamEngine(tmp, max_model_len=8192, block_length=32, mask_token_id=mask_id, threshold=0.9,
                                            gpu_memory_utilization=0.5, enforce_eager=True)
        gen = torch.Generator().manual_seed(0)
        context = torch.randint(0, 151000, (8192,), generator=gen).tolist()
        query = torch.randint(0, 151000, (64,), generator=gen).tolist()
        chunks = [([bos] + context[i:i + 1024])[:1024] for i in range(0, 8192, 1024)]

        def sync_ms(fn):
            torch.cuda.synchronize(device)
            t0 = time.perf_counter()
            r = fn()
            torch.cuda.synchronize(device)
            return r, (time.perf_counter() - t0) * 1e3

        runs = []
        with torch.inference_mode():
            for it in range(out["steps"] + 1):
                (selected, scores, _, _), t_sel = sync_ms(lambda: engine.select_chunks_by_engine([bos], chunks, query, topk_chunks=4))
                prompt = [bos] + [t for ci in selected for t in chunks[ci]] + query
                rec, t_pre = sync_ms(lambda: engine.prefill_to_pd_record(prompt, max_new_tokens=32))
                res, t_dec = sync_ms(lambda: engine.decode_from_pd_record(rec, max_new_tokens=32))
                if it > 0:          # the first request carries torch.compile and autotuning
                    runs.append(dict(draft_and_scoring_ms=t_sel, prefill_ms=t_pre, decode_ms=t_dec, denoise_steps=int(res.n_diff_steps),
                                     new_tokens=len(res.token_ids), selected=[int(i) for i in selected]))
        try:
            engine.close()
        except Exception:
            pass
        mean = {k: sum(r[k] for r in runs) / len(runs) for k in ("draft_and_scoring_ms", "prefill_ms", "decode_ms")}
        total = sum(mean.values())
        out.update(value=32 / (mean["decode_ms"] * 1e-3), ms_per_step=total, phases_ms=mean, runs=runs,
                   e2e={"value": 32 / (total * 1e-3), "unit": "tok/s", "request_latency_ms": total})
    except BaseException as exc:
        out["unavailable"] = f"{type(exc).__name__}: {exc}"[:600]
        out["traceback"] = traceback.format_exc()[-3000:]
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return out


def run_request(args, rank: int, world: int, local_rank: int):
    from prefilling_dllm_b200 import ops
    from prefilling_dllm_b200 import sharded as sharded_mod
    from prefilling_dllm_b200.sharded import ShardedChunkPrefill

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = torch.distributed

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    def max_over_ranks(values):
        t = torch.tensor(values, dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t]

    model = build_dream7b(device)
    steps, warmup = max(1, args.steps), max(3, args.warmup)

    # ---------------- the 8K request: one per rank ----------------
    rt = make_runtime(model, long_ctx=False)
    gen = torch.Generator().manual_seed(rank)
    context = torch.randint(0, 151000, (8192,), generator=gen).tolist()
    query = torch.randint(0, 151000, (64,), generator=gen).tolist()
    new_tokens = rt.max_new_tokens
    timer = PhaseTimer(device)
    timer.wrap(rt, "_selection_query_ids_with_score_target", "draft")
    timer.wrap(rt, "score_chunks_self_information_batched", "scoring")
    timer.wrap(rt, "_denoise_blocks", "decode")

    def request():
        return rt.generate(prefix_ids=rt.bos_ids(), context_ids=context, query_ids=query)

    for _ in range(warmup):
        request()
    ops.check_status(device)
    timer.totals_ms()
    sampler = ClockSampler(local_rank)
    if rank == 0:
        sampler.start()
    calls_before = ops.C_ABI_CALLS
    ms_request, result = timed_requests(request, steps, 0, device, barrier)
    launches = ops.C_ABI_CALLS - calls_before
    phases = {k: v / steps for k, v in timer.totals_ms().items()}
    timer.restore()
    clocks = sampler.stop() if rank == 0 else None
    ops.check_status(device)
    phases["prefill"] = ms_request - sum(phases.values())     # the joint prefill and everything between the wrapped phases
    ms_request, decode_ms = max_over_ranks([ms_request, phases["decode"]])
    denoise_steps = new_tokens - 1                             # random-init weights never reach the threshold: one token per step

    line = None
    if rank == 0:
        peaks = load_peaks()
        line = {
            "metric": "decode_tok_per_s", "value": world * new_tokens / (decode_ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms_request, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "Dream-7B architecture (random init), 8192-token random prefix + 64-token query, chunk 1024 with chunk BOS, "
                                   "draft-self-information scoring at batch 8, top-4, joint full_prompt_mask prefill, block 32, 32 new tokens, "
                                   "threshold 0.9, greedy; one request per step and per GPU through FastDLLMParallelComp.generate",
                       "parallelism": f"dp{world} (one request per rank, no data-path collective)",
                       "l2": "15 GB of weights and the KV pages are streamed again by every forward (> 126 MB L2)"},
            "e2e": {"value": world * new_tokens / (ms_request * 1e-3), "unit": "tok/s", "request_latency_ms": ms_request,
                    "h2d_bytes_per_step": (len(context) + len(query) + 1) * 8 * 2, "d2h_bytes_per_step": new_tokens * 8 + denoise_steps * 4,
                    "what": "host token-id lists in (ids and RoPE positions uploaded), generated ids out as a host list; one 4-byte count read per denoise step"},
            "phases_ms": phases, "denoise_steps": denoise_steps, "ms_per_denoise_step": phases["decode"] / max(1, denoise_steps),
            "selected_chunks": list(result.selected_chunk_indices),
            "gpu_launches": launches, "clocks": clocks,
        }

    # ---------------- kernel shares of one denoise step + roofline of the dominant kernel (rank 0) ----------------
    if rank == 0:
        br = denoise_step_breakdown(model, 32, 4161, device)
        line["kernel_share"] = {"groups_ms": br["groups_ms"], "share": br["share"], "launches": br["launches"], "sum_of_groups_ms": br["sum_of_groups_ms"],
                                "measured_step_ms": line["ms_per_denoise_step"]}
        gbs = br["linear_bytes"] / (br["linear_ms"] * 1e-3) / 1e9
        line["roofline"] = {
            "kernel": "linear_sm100_kernel, the linear layers of one denoise step (32 rows): 4 per layer + LM head",
            "bound": "hbm", "achieved": gbs, "peak": peaks["hbm"], "unit": "GB/s", "frac": gbs / peaks["hbm"],
            "bytes_per_launch": br["linear_bytes"] / br["linear_launches"], "us_per_launch": br["linear_ms"] * 1e3 / br["linear_launches"],
            "launches_timed": br["linear_launches"],
            "traffic": LINEAR_TRAFFIC_OVER_ALGORITHMIC * br["linear_bytes"] / br["linear_launches"],
            "traffic_note": "DRAM bytes of the captured gate/up launch (272.1 MB read + 4.5 MB written for 273.0 MB algorithmic) scaled to the "
                            "step's average launch; every launch of the step streams its weight matrix exactly once the same way",
            "peak_source": peaks["source"] + " (copy bandwidth)"}
    barrier()

    # ---------------- the 32K request, chunks sharded over the ranks ----------------
    rt32 = make_runtime(model, long_ctx=True)
    gen = torch.Generator().manual_seed(32768)
    context32 = torch.randint(0, 151000, (32768,), generator=gen).tolist()
    query32 = torch.randint(0, 151000, (64,), generator=gen).tolist()
    sharded = ShardedChunkPrefill(rt32) if world > 1 else None
    timer = PhaseTimer(device)
    timer.wrap(rt32, "_selection_query_ids_with_score_target", "draft")
    timer.wrap(rt32, "score_chunks_self_information_batched", "scoring")
    timer.wrap(rt32, "_denoise_blocks", "decode")
    timer.wrap(rt32, "_prefill_one_chunk", "chunk_eviction_and_prefill")
    timer.wrap(rt32, "_prefill_chunks_packed", "chunk_eviction_and_prefill")      # one GPU: the selected chunks in packed forwards
    moved = {"all_gather_bytes": 0, "kv_bytes_received": 0}
    if sharded is not None:
        timer.wrap(sharded_mod, "all_gather_chunk_scores", "score_all_gather")
        timer.wrap(sharded_mod, "exchange_chunk_kv", "kv_hand_off")
        inner_exchange = sharded_mod.exchange_chunk_kv

        def counting_exchange(*a, **k):
            got_kv, got_pos = inner_exchange(*a, **k)
            owned = {t.chunk_index for t in a[0] if t.src_rank == k["decode_rank"]}
            moved["kv_bytes_received"] = sum(v.numel() * v.element_size() for ci, v in got_kv.items() if ci not in owned)
            return got_kv, got_pos

        sharded_mod.exchange_chunk_kv = counting_exchange
        moved["all_gather_bytes"] = 4 * world * math.ceil(32 / world)

    def request32():
        if sharded is not None:
            return sharded.generate(prefix_ids=rt32.bos_ids(), context_ids=context32, query_ids=query32, decode_rank=0)
        return rt32.generate(prefix_ids=rt32.bos_ids(), context_ids=context32, query_ids=query32)

    n32 = max(2, min(steps, 3))
    for _ in range(2):
        request32()
    timer.totals_ms()
    ms32, res32 = timed_requests(request32, n32, 0, device, barrier)
    ph32 = {k: v / n32 for k, v in timer.totals_ms().items()}
    timer.restore()
    if sharded is not None:
        sharded_mod.exchange_chunk_kv = inner_exchange
    ops.check_status(device)
    (ms32,) = max_over_ranks([ms32])
    ph_max = max_over_ranks([ph32.get(k, 0.0) for k in ("draft", "scoring", "chunk_eviction_and_prefill", "score_all_gather", "kv_hand_off", "decode")])
    same_selection = None
    if world > 1 and rank == 0:
        # the sharded selection must be the single-GPU selection: rank 0 scores all 32 chunks itself and compares
        chunks, single, _, _, _ = rt32._prepare_candidate_chunks(prefix_ids=rt32.bos_ids(), context_ids=context32, scoring_query_ids=query32)
        same_selection = list(single) == list(res32.selected_chunk_indices)
    barrier()
    if rank == 0:
        names = ("draft", "scoring", "chunk_eviction_and_prefill", "score_all_gather", "kv_hand_off", "decode")
        line["request_32k"] = {
            "workload": "Dream-7B architecture, 32768-token random prefix (32 chunks of 1024) + 64-token query, top-8, token_capacity 256, "
                        "chunk_query cache mode, 64 new tokens (2 blocks); " + (f"chunk scoring and chunk prefill sharded over {world} ranks, decode on rank 0"
                                                                                 if world > 1 else "one GPU"),
            "scaling": "strong", "request_latency_ms": ms32, "requests_timed": n32, "decode_tok_per_s": 64 / (ph_max[5] * 1e-3),
            "phases_ms_max_over_ranks": dict(zip(names, ph_max)), "selected_chunks": list(res32.selected_chunk_indices),
            "selection_equals_single_gpu": same_selection, "score_all_gather_bytes": moved["all_gather_bytes"],
            "kv_bytes_received_by_decode_rank": moved["kv_bytes_received"],
        }

    # ---------------- op-level records ----------------
    del rt, rt32
    op_main = op_decode_attention(200, 3, rank, world, device, with_e2e=(rank == 0))
    if rank == 0:
        del model
        torch.cuda.empty_cache()
        line["ops"] = {"decode_attention_8_requests": op_main, "decode_attention_1_request_32_rows": op_decode_rows(device, 5),
                       "mha_decode_16_requests": op_mha_decode(16, 100, rank, device),
                       "prefill_attention": op_prefill_attention(device, 50), "linear": op_linear(device, 5),
                       "reference_triton_same_gpu": reference_triton_on_this_gpu(device)}
        if world == 1:
            line["cpu_baseline"], line["toy_same_config"] = cpu_toy_baseline(), gpu_toy_same_config(device)
            if not args.skip_reference_engine:
                # the reference's own GPU code on the same request, on this GPU (about a minute each: checkpoint, load, warm-up):
                # its PD engine, and its eval class (device=cuda) over the restated plain-PyTorch plug-in model
                keep = ("value", "unit", "ms_per_step", "phases_ms", "e2e", "unavailable", "config")
                for key, fn in (("reference_engine_same_gpu", run_reference_engine_8k), ("reference_class_same_gpu", run_reference_class_8k)):
                    gc.collect()
                    torch.cuda.empty_cache()
                    ref = fn(args, local_rank)
                    torch.set_default_device("cpu")            # the reference's model runner changes both while it builds its model
                    torch.set_default_dtype(torch.float32)
                    line[key] = {k: ref[k] for k in keep if k in ref}
                    if "value" in ref:
                        line[key]["this_build_over_reference"] = {"decode_tok_per_s": line["value"] / ref["value"],
                                                                  "request_latency": ref["ms_per_step"] / line["ms_per_step"]}
    barrier()
    return line


# (dram__bytes_read.sum + dram__bytes_write.sum) / algorithmic bytes of one linear_sm100_kernel launch at 32 rows: the ncu capture of the
# gate/up projection (profiles/linear_sm100_kernel_gate_up_32_rows.md) read 272.1 MB and wrote 4.5 MB for 273.0 MB of weights, rows and outputs
LINEAR_TRAFFIC_OVER_ALGORITHMIC = 276.6 / 273.0

# ---- the reference's CPU path on the toy, and this runtime on the same toy ----------------------------------------------------
def _toy_setup(tmp):
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import make_golden

    ckpt = os.path.join(tmp, "ckpt_toy")
    make_golden.write_toy_checkpoint(ckpt)
    context, query = make_golden.toy_inputs()
    return ckpt, context, query, dict(make_golden.README_FLAGS)


TOY_WORKLOAD = ("CPU toy: Dream architecture, 2 layers, hidden 256, 4/2 heads of 64, MLP 688, vocabulary 1024, fp32, seeded init; 4096 random "
                "context ids + 32-token query, chunk 512 with chunk BOS, top-4, 4 draft tokens / 1 round, block 32, 32 new tokens, threshold 0.9")


def cpu_toy_baseline(repeats: int = 3, warmup: int = 1):
    """One toy request on the host cores: the reference's own class when it is staged under oracle/_ref, else the chained CPU
    restatement. A bounded sample by construction: the toy is the only configuration the reference can run on a CPU in seconds."""
    import tempfile

    from oracle import build_ref, toy_request

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    with tempfile.TemporaryDirectory() as tmp:
        ckpt, context, query, flags = _toy_setup(tmp)
        try:
            for _ in range(max(1, warmup)):
                toy_request.run_reference_class(ckpt, context, query, flags)    # warm-up
            got = toy_request.run_reference_class(ckpt, context, query, flags, repeats=repeats)
            kind = "reference"
        except build_ref.RefUnavailable:
            from oracle.contract_model.model.modeling_dream import DreamModel

            model = DreamModel.from_pretrained(ckpt).eval()
            toy_request.run_port(model, context, query, flags)
            got = toy_request.run_port(model, context, query, flags)
            kind = "port"
    return {"value": got["decode_tok_per_s"], "unit": "tok/s", "cores": cores, "kind": kind,
            "sample": f"{TOY_WORKLOAD}; whole request {got['seconds']['total']:.2f} s, decode phase {got['seconds']['decode']:.2f} s",
            "request_latency_ms": got["seconds"]["total"] * 1e3, "phases_ms": {k: v * 1e3 for k, v in got["seconds"].items() if k != "total"},
            "sequences": got["sequences"], "selected_chunks": got["selected"]}


def gpu_toy_same_config(device):
    """This runtime on the same toy, fp32, so that the CPU figure has a same-configuration counterpart."""
    import tempfile

    from prefilling_dllm_b200.parallelcomp import load_fastdllm_parallelcomp

    with tempfile.TemporaryDirectory() as tmp:
        ckpt, context, query, flags = _toy_setup(tmp)
        rt = load_fastdllm_parallelcomp(pretrained=ckpt, device=str(device), dtype="float32", **flags)
        timer = PhaseTimer(device)
        timer.wrap(rt, "_denoise_blocks", "decode")

        def request():
            return rt.generate(prefix_ids=rt.bos_ids(), context_ids=context, query_ids=query)

        for _ in range(3):
            request()
        timer.totals_ms()
        ms, result = timed_requests(request, 5, 0, device, lambda: torch.cuda.synchronize(device))
        decode_ms = timer.totals_ms()["decode"] / 5
        timer.restore()
    return {"workload": TOY_WORKLOAD, "value": len(result.sequences) / (decode_ms * 1e-3), "unit": "tok/s", "request_latency_ms": ms,
            "decode_ms": decode_ms, "sequences": list(result.sequences), "selected_chunks": list(result.selected_chunk_indices)}


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return None
    steps, warmup = max(1, min(args.steps, 200)), max(1, min(args.warmup, 50))      # a toy request takes a fraction of a second
    t0 = time.perf_counter()
    base = cpu_toy_baseline(repeats=steps, warmup=warmup)
    wall = time.perf_counter() - t0
    return {
        "impl": "reference", "metric": "decode_tok_per_s", "value": base["value"], "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": base["request_latency_ms"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": TOY_WORKLOAD, "note": "the one configuration the reference's CPU path finishes in seconds; "
                                       "the native arm reports this runtime on the same toy as toy_same_config", "wall_s": wall},
        "cpu_baseline": base, "e2e": {"value": 32 / (base["request_latency_ms"] * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
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
    # llada8b_decode_batch: LLaDA-8B architecture (32 MHA heads, un-shifted logits, 16 concurrent requests),
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



def run_byte_kernels(args, local_rank: int):
    """Achieved HBM rate of each byte-moving kernel of the path at Dream-7B request shapes, one GPU.
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

    # row ops of the transformer block at the two shapes of a request: one denoise block (32 rows) and the scoring prefill (8744 rows)
    hq, hidden = 28, 3584
    ln_w = torch.ones(hidden, device=device, dtype=torch.bfloat16)
    for n_rows, sets in ((32, 16), (8744, 4)):
        xs = [torch.randn(n_rows, hidden, device=device, dtype=torch.bfloat16, generator=g) for _ in range(sets)]
        ds = [torch.randn(n_rows, hidden, device=device, dtype=torch.bfloat16, generator=g) for _ in range(sets)]
        timed("add_rmsnorm_vec_kernel (residual add + RMSNorm)", f"{n_rows} rows x 3584 bf16", n_rows * hidden * 2 * 4,      # x and delta read, x and out written
              lambda i, xs=xs, ds=ds: ops.add_rmsnorm(xs[i], ln_w, 1e-6, ds[i]), sets)
        qkvs = [torch.randn(n_rows, hq + 2 * hkv, d, device=device, dtype=torch.bfloat16, generator=g) for _ in range(sets)]
        cos = torch.randn(n_rows, d, device=device, dtype=torch.bfloat16, generator=g)
        rs_k = torch.zeros(40, page, hkv, d, device=device, dtype=torch.bfloat16)
        rs_v = torch.zeros_like(rs_k)
        rs_slots = torch.randperm(40 * page, device=device, generator=g)[:n_rows].to(torch.int32)
        timed("rope_store_kernel (RoPE of q, k in place + page write of k, v)", f"{n_rows} rows x (28 + 2 x 4) heads x 128 bf16",
              n_rows * ((hq + hkv) * d * 2 * 2 + 2 * hkv * d * 2 * 2 + 2 * d * 2),
              lambda i, qkvs=qkvs: ops.rope_store(qkvs[i], cos, cos, hq, hkv, rs_k, rs_v, rs_slots), sets)
        del xs, ds, qkvs

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



def run_op(args, rank: int, world: int, local_rank: int):
    """`--workload op`: the op-level decode attention alone, one replica per rank (weak scaling, no collective)."""
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    sampler = ClockSampler(local_rank)
    if rank == 0:
        sampler.start()
    rec = op_decode_attention(args.steps, args.warmup, rank, world, device)
    t = torch.tensor([rec["us_per_launch"], rec["host_buffers"]["us_per_step"]], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    clocks = sampler.stop() if rank == 0 else None
    if rank != 0:
        return None
    us, e2e_us = float(t[0]), float(t[1])
    return {"metric": "decode_attention_tok_per_s", "value": world * NUM_REQ * ROWS / (us * 1e-6), "unit": "tok/s", "n_gpus": world,
            "steps": rec["launches"], "warmup": max(3, args.warmup), "ms_per_step": us * 1e-3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": OP_WORKLOAD, "parallelism": f"dp{world} (replicas over requests, no data-path collective)", "l2": rec["l2"]},
            "roofline": rec["roofline"],
            "e2e": {"value": world * NUM_REQ * ROWS / (e2e_us * 1e-6), "unit": "tok/s", "h2d_bytes_per_step": rec["host_buffers"]["h2d_bytes_per_step"],
                    "d2h_bytes_per_step": rec["host_buffers"]["d2h_bytes_per_step"], "ms_per_step": e2e_us * 1e-3},
            "gpu_launches": rec["launches"], "clocks": clocks}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--workload", default="request",
                    choices=["request", "request_once", "full_reencode", "reference_engine_8k", "reference_class_8k", "op", "op_mha_decode", "op_decode_rows", "op_prefill", "linear", "byte_kernels", "dream7b_decode_batch",
                             "llada8b_decode_batch"],
                    help="request (default): the 8K request per GPU + the sharded 32K request + op-level records; the others run one piece alone")
    ap.add_argument("--shape", default="", help="--workload linear: run one shape only, e.g. gate_up_m32 (for a profiler capture)")
    ap.add_argument("--skip-reference-engine", action="store_true",
                    help="default workload at N = 1: do not run the reference's own GPU engine on the same request at the end")
    ap.add_argument("--ctx", type=int, default=8192, help="--workload full_reencode: context length (8192 or 32768)")
    ap.add_argument("--concurrent", type=int, default=16, help="requests per GPU that share a denoise step (decode_batch workloads, op_mha_decode)")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    # stdout carries the ONE JSON line and nothing else: whatever libraries print while they load (some log to stdout) goes
    # to stderr, at the file-descriptor level so that native code is covered too
    sys.stdout.flush()
    result_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    sys.stdout = sys.stderr

    def emit(line):
        if line is not None:
            result_out.write(json.dumps(line) + "\n")
            result_out.flush()

    if args.impl == "reference":
        emit(run_reference(args, rank, world))
        return

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device: the product path has no CPU fallback")
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        device = torch.device("cuda", local_rank)
        torch.cuda.set_device(device)
        if args.workload == "request":
            line = run_request(args, rank, world, local_rank)
        elif args.workload == "op":
            line = run_op(args, rank, world, local_rank)
        elif args.workload == "op_mha_decode":
            line = op_mha_decode(max(1, args.concurrent), args.steps, rank, device) if rank == 0 else None
        elif args.workload == "op_prefill":
            line = op_prefill_attention(device, args.steps) if rank == 0 else None
        elif args.workload == "linear":
            line = op_linear(device, args.steps, args.shape) if rank == 0 else None
        elif args.workload == "op_decode_rows":
            line = op_decode_rows(device, args.steps) if rank == 0 else None
        elif args.workload == "reference_class_8k":
            line = run_reference_class_8k(args, local_rank) if rank == 0 else None
        elif args.workload == "reference_engine_8k":
            line = run_reference_engine_8k(args, local_rank) if rank == 0 else None
        elif args.workload == "full_reencode":
            line = run_full_reencode(args, local_rank) if rank == 0 else None
        elif args.workload == "request_once":
            line = run_request_once(local_rank) if rank == 0 else None
        elif args.workload == "byte_kernels":
            line = run_byte_kernels(args, local_rank) if rank == 0 else None
        else:
            line = run_decode_batch(args, rank, world, local_rank)
        emit(line)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
