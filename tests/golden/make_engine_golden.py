"""Golden vectors of the reference's PD ENGINE, produced by the unmodified reference code on a GPU machine.

`FastDLLMDreamEngine` (prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py:170) builds a model runner that initialises
CUDA and NCCL, so unlike the eval class (make_golden.py) it cannot run on a CPU box. This script runs it where a GPU is
present, from the copy staged under oracle/_ref/engine (oracle/build_ref.py; byte-for-byte, git-ignored), over the seeded toy
checkpoint of make_golden.py, and records what the engine-side parity tests compare:

  * the prefill/decode split: first token, last-context logit, denoised ids and step count of `prefill_to_pd_record` →
    `decode_from_pd_record` for three prompts, a checksum of the snapshot KV, and the same request through
    `generate_token_ids`;
  * post-hoc eviction with head-independent keep indices;
  * the selection twins: the engine's draft, `select_chunks_by_engine` (scores, selection, label mask),
    `score_chunk_self_information_engine` under the causal and query_to_chunk masks,
    `compute_prompt_keep_indices_per_layer_per_head`, `generate_token_ids_from_chunk_local_kv`.

    python oracle/build_ref.py --reference <checkout>          # where the checkout exists
    python tests/golden/make_engine_golden.py --out tests/golden/engine_reference.json     # on a machine with a GPU

Model dtype. The fixture is made with the checkpoint declared float64 and the reference's `sdpa` attention backend. In float32
the reference engine does not compute the model: its RMSNorm (layers/layernorm.py:18-41) converts with `x.to(torch.float32)`,
which for a float32 input is the SAME tensor, and then normalises in place — so the residual stream is overwritten by its own
normalised copy in every layer (in bfloat16, the dtype it is deployed in, the conversion copies and the arithmetic is the
model's). Declared float64, every conversion copies again: norms and RoPE are evaluated in float32 as in deployment, the
products in float64, and the result is the model's arithmetic to ~1e-7 — what a float32 restatement can be held to bit for
bit on discrete outputs. `--dtype float32` reproduces the aliasing artefact (first token 989 instead of 290 on the first prompt).

If the reference engine cannot be constructed there, the script writes {"unavailable": "<exception>"} so that the reason
is on record; the tests then keep oracle/engine_flow.py as their checker.
"""

import argparse
import json
import os
import shutil
import sys
import tempfile
import traceback

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import make_golden  # noqa: E402

BOS, MASK, BLOCK = make_golden.BOS, make_golden.MASK, 32


def prompt(n=600, seed=3):
    g = torch.Generator().manual_seed(seed)
    return [BOS] + torch.randint(3, 1000, (n - 1,), generator=g).tolist()


def toy_checkpoint_for_the_engine(path: str, dtype: str) -> None:
    """The toy checkpoint plus what the engine's loader wants: an auto_map to the Dream configuration class the reference
    vendors (staged copy), since its Config resolves the model through AutoConfig with trust_remote_code."""
    from oracle import build_ref

    make_golden.write_toy_checkpoint(path)
    shutil.copyfile(os.path.join(build_ref.REF_DIR, "engine", "configuration_dream.py"), os.path.join(path, "configuration_dream.py"))
    cfg_path = os.path.join(path, "config.json")
    with open(cfg_path) as handle:
        cfg = json.load(handle)
    cfg["auto_map"] = {"AutoConfig": "configuration_dream.DreamConfig"}
    cfg["architectures"] = ["DreamModel"]
    cfg["torch_dtype"] = dtype
    with open(cfg_path, "w") as handle:
        json.dump(cfg, handle)


def record(engine) -> dict:
    out = {}
    # ---- prefill / decode split ----
    runs = []
    for n, seed in ((600, 3), (500, 9), (257, 11)):
        ids = prompt(n, seed)
        rec = engine.prefill_to_pd_record(ids, max_new_tokens=BLOCK)
        snap = engine.snapshot_pd_record_kv(rec)
        item = dict(prompt_len=n, seed=seed, first_token_id=int(rec.first_token_id), prompt_len_record=int(rec.prompt_len),
                    suffix_positions=[int(p) for p in rec.suffix_positions],
                    last_context_logit=[float(x) for x in rec.last_context_logit.float().reshape(-1).tolist()],
                    k_abs_sum=[float(k.float().abs().sum()) for k in snap.k_by_layer],
                    v_abs_sum=[float(v.float().abs().sum()) for v in snap.v_by_layer],
                    k_shape=list(snap.k_by_layer[0].shape))
        res = engine.decode_from_pd_record(rec, max_new_tokens=BLOCK)
        item.update(token_ids=[int(t) for t in res.token_ids], n_diff_steps=int(res.n_diff_steps))
        fused = engine.generate_token_ids(ids, max_new_tokens=BLOCK)
        item.update(fused_token_ids=[int(t) for t in fused.token_ids])
        runs.append(item)
    out["pd_split"] = runs
    # ---- post-hoc eviction with head-independent keep indices ----
    ids = prompt(600, 7)
    keep = [0] + list(range(1, 600, 3))
    nested = [[list(keep) for _ in range(2)] for _ in range(2)]
    rec = engine.prefill_to_pd_record(ids, max_new_tokens=BLOCK, prompt_keep_indices_per_layer_per_head=nested, active_prompt_positions=keep)
    item = dict(prompt_len=600, seed=7, keep=keep, kv_mode=str(rec.kv_mode), prompt_len_record=int(rec.prompt_len),
                full_prompt_len=int(rec.full_prompt_len), first_token_id=int(rec.first_token_id),
                suffix_positions=[int(p) for p in rec.suffix_positions])
    res = engine.decode_from_pd_record(rec, max_new_tokens=BLOCK)
    item.update(token_ids=[int(t) for t in res.token_ids], n_diff_steps=int(res.n_diff_steps))
    out["posthoc_eviction"] = item
    # ---- selection twins ----
    context, query = make_golden.toy_inputs()
    chunks = []
    for c in make_golden_split(context, 512):
        c = [BOS] + list(c)
        chunks.append(c[:512])
    draft_ids, draft_mask = engine.generate_partial_draft_rounds_for_selection([BOS] + query, max_new_tokens=4, partial_rounds=1)
    selected, scores, sel_ids, mask = engine.select_chunks_by_engine([BOS], chunks, query, topk_chunks=4)
    selection = [int(t) for t in sel_ids]
    label_mask = None if mask is None else [bool(m) for m in mask]
    one = engine.score_chunk_self_information_engine([BOS], chunks[2], selection, score_token_mask=label_mask)
    q2c = engine.score_chunk_self_information_engine([BOS], chunks[2], selection, score_token_mask=label_mask,
                                                     score_attention_mask="query_to_chunk")
    out["selection"] = dict(draft_ids=[int(t) for t in draft_ids], draft_mask=[bool(m) for m in draft_mask],
                            selected=[int(i) for i in selected], scores={str(k): float(v) for k, v in scores.items()},
                            selection_query_ids=selection, score_token_mask=label_mask, chunk2_causal=float(one), chunk2_query_to_chunk=float(q2c))
    a, b = chunks[selected[0]], chunks[selected[1]]
    spans = [dict(chunk_ids=a, start=1, end=1 + len(a)), dict(chunk_ids=b, start=1 + len(a), end=1 + len(a) + len(b))]
    full_len = 1 + len(a) + len(b) + len(query)
    keep_ph, meta = engine.compute_prompt_keep_indices_per_layer_per_head(full_prompt_len=full_len, prefix_ids=[BOS], chunk_spans=spans,
                                                                         query_ids=query, token_capacity=128)
    out["per_head_keep"] = dict(full_prompt_len=full_len, keep=[[[int(i) for i in head] for head in layer] for layer in keep_ph],
                                meta=[{k: (int(v) if isinstance(v, (int, bool)) else v) for k, v in m.items() if isinstance(v, (int, float, str, bool))}
                                      for m in meta])
    # ---- chunk-local KV generate ----
    two = chunks[:2]
    keeps = [[0] + list(range(5, 512, 4)), [0] + list(range(2, 512, 4))]
    chunk_pos = [list(range(1, 513)), list(range(1, 513))]
    q_pos = list(range(513, 513 + len(query)))
    nested = [[[list(k), list(k)] for _ in range(2)] for k in keeps]
    res = engine.generate_token_ids_from_chunk_local_kv(prefix_ids=[BOS], prefix_positions=[0], chunk_ids_list=two, chunk_positions_list=chunk_pos,
                                                        chunk_keep_indices_per_layer_per_head=nested, query_ids=query, query_positions=q_pos,
                                                        local_query_ids=query[-8:], max_new_tokens=BLOCK)
    out["chunk_local"] = dict(keeps=keeps, token_ids=[int(t) for t in res.token_ids], n_diff_steps=int(res.n_diff_steps))
    out["sparse_and_delta"] = record_sparse_and_delta(engine)
    out["sampling"] = record_sampling(engine)
    out["per_head_keep_variants"] = record_keep_variants(engine, spans, full_len, query)
    return out


def per_head_keep_lists(n: int = 600, kept: int = 200):
    """[layer][head] ascending keep indices of equal length that differ per layer and head (their union is what a sparse
    prefill may attend)."""
    return [[([0] + list(range(1 + (h + 2 * layer) % 3, n, 3)))[:kept] for h in range(2)] for layer in range(2)]


SPARSE_DELTA_CASES = {
    "sparse_prefill": dict(prefill_sparse_mode="eviction_mask"),
    "sparse_prefill_delta_left": dict(prefill_sparse_mode="eviction_mask", prefill_delta_mode="s4_left3"),
    "sparse_prefill_delta_both": dict(prefill_sparse_mode="eviction_mask", prefill_delta_mode="s4_left3", prefill_delta_stride=4,
                                      prefill_delta_left=1, prefill_delta_right=2, prefill_delta_direction="both", prefill_delta_scale=0.5),
    "sparse_prefill_delta_right": dict(prefill_sparse_mode="eviction_mask", prefill_delta_mode="s4_left3", prefill_delta_stride=4,
                                       prefill_delta_right=3, prefill_delta_direction="right"),
    "posthoc_decode_delta": dict(decode_delta_mode="s4_left3"),
    "posthoc_decode_delta_stride8": dict(decode_delta_mode="s4_left3", decode_delta_stride=8, decode_delta_left=5, decode_delta_scale=0.5),
}


def record_sparse_and_delta(engine) -> dict:
    """The engine's sparse prefill over an eviction mask (with and without the strided delta correction) and its decode-time
    delta correction against a full-KV reservoir (fastdllm_engine.py:1924-2080, layers/attention/attention_v4.py:86-289)."""
    ids = prompt(600, 13)
    nested = per_head_keep_lists()
    active = nested[0][0]
    cases = {}
    for name, kwargs in SPARSE_DELTA_CASES.items():
        try:
            rec = engine.prefill_to_pd_record(ids, max_new_tokens=BLOCK, prompt_keep_indices_per_layer_per_head=nested,
                                              active_prompt_positions=active, **kwargs)
            item = dict(kv_mode=str(rec.kv_mode), prompt_len_record=int(rec.prompt_len), full_prompt_len=int(rec.full_prompt_len),
                        first_token_id=int(rec.first_token_id), suffix_positions=[int(p) for p in rec.suffix_positions],
                        last_context_logit=[float(x) for x in rec.last_context_logit.float().reshape(-1).tolist()],
                        n_prompt_pages=len(rec.prompt_page_ids))
            res = engine.decode_from_pd_record(rec, max_new_tokens=BLOCK)
            item.update(token_ids=[int(t) for t in res.token_ids], n_diff_steps=int(res.n_diff_steps))
        except Exception as exc:  # a mode the reference itself cannot run is recorded as such
            item = dict(error=f"{type(exc).__name__}: {exc}"[:300])
        cases[name] = item
    return dict(prompt_len=600, seed=13, cases=cases)


KEEP_VARIANTS = {
    "avgpool": dict(token_score_pooling="avgpool"),
    "no_pooling_mean_reduce": dict(token_score_pooling="none", token_score_reduce="mean"),
    "keep_low": dict(token_score_keep="low"),
    "chunk_to_query_full_mask": dict(token_score_direction="chunk_to_query", token_attention_mask="full"),
    "bidirectional_full_mask_avgpool": dict(token_score_direction="bidirectional", token_attention_mask="full", token_score_pooling="avgpool",
                                            token_score_pool_kernel=5),
    "two_layers_last": dict(token_score_layers=2, token_score_layer_mode="last", token_attention_mask="query_to_chunk"),
}


def record_keep_variants(engine, spans, full_len, query) -> dict:
    """compute_prompt_keep_indices_per_layer_per_head (fastdllm_engine.py:1325-1563) off its defaults: pooling, reduce, keep-low, the
    chunk->query and bidirectional directions (_engine_chunk_attention_head_scores :1230-1323), the layer window."""
    cases = {}
    for name, kwargs in KEEP_VARIANTS.items():
        try:
            keep, meta = engine.compute_prompt_keep_indices_per_layer_per_head(full_prompt_len=full_len, prefix_ids=[BOS], chunk_spans=spans,
                                                                               query_ids=query, token_capacity=128, **kwargs)
            cases[name] = dict(keep=[[[int(i) for i in head] for head in layer] for layer in keep],
                               kept=[int(m["kept_tokens"]) for m in meta])
        except Exception as exc:
            cases[name] = dict(error=f"{type(exc).__name__}: {exc}"[:300])
    return dict(full_prompt_len=full_len, cases=cases)


SAMPLING_CASES = {
    "top_k_1": dict(top_k=1),                              # every probability is 1: the whole block in one step
    "top_k_2": dict(top_k=2),
    "top_p_half": dict(top_p=0.5),
    "top_k_4_top_p_0.8": dict(top_k=4, top_p=0.8),
    "temperature_0.7_top_k_8": dict(temperature=0.7, top_k=8),
}


def record_sampling(engine) -> dict:
    """The engine's sampler settings (fastdllm_engine.py:1658-1681, :2143-2157), switched on the one engine between requests:
    filters at temperature 0 change the confidences the threshold rule sees (several slots per step even with random weights);
    the positive temperature draws from the global generator, seeded before the request."""
    ids = prompt(500, 21)
    saved = (engine.temperature, engine.top_k, engine.top_p)
    cases = {}
    try:
        for name, kwargs in SAMPLING_CASES.items():
            engine.temperature, engine.top_k, engine.top_p = float(kwargs.get("temperature", 0.0)), kwargs.get("top_k"), kwargs.get("top_p")
            torch.manual_seed(77)
            try:
                rec = engine.prefill_to_pd_record(ids, max_new_tokens=BLOCK)
                first = int(rec.first_token_id)
                res = engine.decode_from_pd_record(rec, max_new_tokens=BLOCK)
                cases[name] = dict(first_token_id=first, token_ids=[int(t) for t in res.token_ids], n_diff_steps=int(res.n_diff_steps))
            except Exception as exc:
                cases[name] = dict(error=f"{type(exc).__name__}: {exc}"[:300])
    finally:
        engine.temperature, engine.top_k, engine.top_p = saved
    return dict(prompt_len=500, seed=21, cases=cases)


def make_golden_split(ids, size):
    return [ids[i:i + size] for i in range(0, len(ids), size)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "engine_reference.json"))
    ap.add_argument("--dtype", default="float64", choices=["float64", "float32", "bfloat16"],
                    help="model dtype of the reference engine (see the module docstring for why float64)")
    ap.add_argument("--attention-backend", default="sdpa", choices=["sdpa", "flex"],
                    help="the reference's PREFILLING_DLLM_ENGINE_ATTENTION_BACKEND (attention_v4.py:38); flex has no float64 kernel")
    args = ap.parse_args()
    os.environ["PREFILLING_DLLM_ENGINE_ATTENTION_BACKEND"] = args.attention_backend
    golden = {"config": dict(make_golden.TOY), "dtype": args.dtype, "attention_backend": args.attention_backend, "block_length": BLOCK,
              "threshold": 0.9}
    tmp = tempfile.mkdtemp()
    try:
        from oracle import build_ref

        module = build_ref.load_reference_engine()
        ckpt = os.path.join(tmp, "ckpt_toy_engine")
        toy_checkpoint_for_the_engine(ckpt, args.dtype)
        engine = module.FastDLLMDreamEngine(ckpt, max_model_len=8192, block_length=BLOCK, mask_token_id=MASK, threshold=0.9,
                                            gpu_memory_utilization=0.05, enforce_eager=True)
        try:
            with torch.inference_mode():
                golden.update(record(engine))
        finally:
            try:
                engine.close()
            except Exception:  # the runner's exit path tears down process groups it may not own
                pass
    except BaseException as exc:  # the reason goes on record; the tests fall back to oracle/engine_flow.py
        golden["unavailable"] = f"{type(exc).__name__}: {exc}"
        golden["traceback"] = traceback.format_exc()[-4000:]
        print(golden["traceback"], file=sys.stderr)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    with open(args.out, "w") as handle:
        json.dump(golden, handle)
    print("wrote", args.out, os.path.getsize(args.out), "bytes;", "unavailable: " + golden["unavailable"] if "unavailable" in golden else "ok")


if __name__ == "__main__":
    main()
