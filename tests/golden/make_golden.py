"""Generates tests/golden/toy_reference.json by running the UNMODIFIED reference class on CPU.

Run where the reference checkout exists:  python tests/golden/make_golden.py --reference /path/to/reference
(or set PDLLM_REFERENCE_ROOT)
It needs only CPU. The reference's model plug-in (Fast-dLLM v1, absent from the reference tree) is supplied by
oracle/contract_model; everything else — chunking, chunk BOS, draft rounds, self-information scoring, ranking,
token eviction, position bookkeeping, block denoising — is the reference's own code
(prefilling_dllm_eval/fastdllm_parallelcomp.py). The JSON it writes is what pins oracle/hotpath.py and the
GPU path; the GPU box never needs the reference.

Workload = the CPU-runnable toy: Dream architecture, 2 layers, hidden 256, 4 query / 2 KV heads, head_dim 64,
MLP 688, vocab 1024, RoPE theta 1e6, fp32, seeded N(0, 0.02) init; 4096 uniform random context ids (seed 0) and a
32-token query; chunk_size 512 with chunk BOS, topk 4, 4 draft tokens / 1 partial round, block 32, 32 new tokens,
threshold 0.9, greedy. Token ids: BOS 1, EOS 2, MASK 1023; sampled ids avoid them.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

TOY = dict(vocab_size=1024, hidden_size=256, intermediate_size=688, num_hidden_layers=2, num_attention_heads=4,
           num_key_value_heads=2, max_position_embeddings=32768, rope_theta=1000000.0, rms_norm_eps=1e-6,
           initializer_range=0.02, mask_token_id=1023, pad_token_id=0, bos_token_id=1, eos_token_id=2)
BOS, EOS, MASK = 1, 2, 1023
# The same flow at the head shape the tensor-core attention kernel serves (head_dim 128, GQA group 2): 2 layers, hidden 512,
# 4 query / 2 KV heads, MLP 1376, vocabulary 4096; MASK is the last id. Run in fp32 and in bf16 by the reference.
TOY128 = dict(vocab_size=4096, hidden_size=512, intermediate_size=1376, num_hidden_layers=2, num_attention_heads=4,
              num_key_value_heads=2, max_position_embeddings=32768, rope_theta=1000000.0, rms_norm_eps=1e-6,
              initializer_range=0.02, mask_token_id=4095, pad_token_id=0, bos_token_id=1, eos_token_id=2)


def toy_inputs(context_len=4096, query_len=32, seed=0, vocab=1024):
    g = torch.Generator().manual_seed(seed)
    context = torch.randint(3, vocab - 1, (context_len,), generator=g).tolist()
    query = torch.randint(3, vocab - 1, (query_len,), generator=g).tolist()
    return context, query


def write_toy_checkpoint(path: str, seed: int = 0, config: dict = None) -> None:
    """config.json + seeded-init model.safetensors + a word-level tokenizer over the vocabulary."""
    TOY = dict(config or globals()["TOY"])
    MASK = TOY["mask_token_id"]
    from safetensors.torch import save_file
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import Whitespace

    from oracle.contract_model.model.configuration_dream import DreamConfig
    from oracle.contract_model.model.modeling_dream import DreamModel, init_weights_

    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as handle:
        json.dump(dict(TOY, model_type="Dream", torch_dtype="float32"), handle)
    model = DreamModel(DreamConfig(**TOY))
    init_weights_(model, seed)
    save_file({k: v.contiguous() for k, v in model.state_dict().items()}, os.path.join(path, "model.safetensors"))
    vocab = {f"t{i}": i for i in range(TOY["vocab_size"])}
    vocab.pop("t1"), vocab.pop("t2"), vocab.pop(f"t{MASK}"), vocab.pop("t0")
    vocab.update({"<pad>": 0, "<bos>": BOS, "<eos>": EOS, "<mask>": MASK})
    tok = Tokenizer(WordLevel(vocab, unk_token="<pad>"))
    tok.pre_tokenizer = Whitespace()
    tok.save(os.path.join(path, "tokenizer.json"))
    with open(os.path.join(path, "tokenizer_config.json"), "w") as handle:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "bos_token": "<bos>", "eos_token": "<eos>",
                   "mask_token": "<mask>", "pad_token": "<pad>", "unk_token": "<pad>"}, handle)


README_FLAGS = dict(  # the reference README's canonical long-context flags (README.md:117-145)
    cache_build_mode="full_prompt_mask", score_mode="draft_self_information", score_draft_tokens=4,
    score_draft_partial_rounds=1, score_context_mode="single_chunk", score_attention_mask="causal", score_batch_size=8,
    chunk_position_mode="continuous", query_position_mode="after_selected_chunks", token_capacity=0,
    chunk_size=512, topk_chunks=4, block_length=32, max_new_tokens=32, threshold=0.9, temperature=0.0,
)


def load_reference(reference_root: str, ckpt: str, dtype: str = "float32", **flags):
    eval_dir = os.path.join(reference_root, "prefilling_dllm_eval")
    if eval_dir not in sys.path:
        sys.path.insert(0, eval_dir)
    import fastdllm_parallelcomp as ref  # the reference module, unmodified

    runtime = ref.load_fastdllm_parallelcomp(
        pretrained=ckpt, fastdllm_dream_dir=os.path.join(ROOT, "oracle", "contract_model"), device="cpu", dtype=dtype,
        trust_remote_code=False, **flags)
    return ref, runtime


def record_run(runtime, context, query, *, capture_steps=True):
    """generate() with the intermediate quantities captured by wrapping bound methods (no reference edits)."""
    rec = {}
    orig_draft = runtime.generate_partial_draft_rounds_from_cache
    orig_keep = runtime._keep_positions_for_chunk
    orig_keep_ph = runtime._keep_positions_per_layer_per_head_for_chunk
    orig_tok_scores = runtime.query_attention_token_scores
    orig_denoise = runtime._denoise_block_confidence_threshold
    orig_fwd_replace = runtime._forward_generation_block_replace
    orig_selection = runtime._selection_query_ids_with_score_target

    def selection(prefix_ids, scoring_query_ids):
        ids, count, mask = orig_selection(prefix_ids, scoring_query_ids)
        rec["selection_query_ids"] = list(ids)
        rec["score_token_mask"] = None if mask is None else [bool(x) for x in mask]
        return ids, count, mask

    def draft(**kw):
        ids, mask = orig_draft(**kw)
        rec["draft_ids"], rec["draft_confirmed"] = list(ids), list(mask)
        return ids, mask

    def keep(prefix_ids, chunk_ids, query_ids):
        out = orig_keep(prefix_ids, chunk_ids, query_ids)
        rec.setdefault("keep_positions", []).append(list(out))
        return out

    def keep_ph(prefix_ids, chunk_ids, query_ids):
        out = orig_keep_ph(prefix_ids, chunk_ids, query_ids)
        rec.setdefault("keep_positions_per_head", []).append([t.tolist() for t in out])
        return out

    def tok_scores(*a, **kw):
        out = orig_tok_scores(*a, **kw)
        rec.setdefault("token_scores", []).append([float(x) for x in out.tolist()])
        return out

    steps = []

    def fwd_replace(block_ids, **kw):
        logits, cache = orig_fwd_replace(block_ids, **kw)
        if capture_steps:
            steps.append(block_ids[0].tolist())
        return logits, cache

    runtime.generate_partial_draft_rounds_from_cache = draft
    runtime._keep_positions_for_chunk = keep
    runtime._keep_positions_per_layer_per_head_for_chunk = keep_ph
    runtime.query_attention_token_scores = tok_scores
    runtime._forward_generation_block_replace = fwd_replace
    runtime._selection_query_ids_with_score_target = selection
    try:
        result = runtime.generate(prefix_ids=runtime.bos_ids(), context_ids=context, query_ids=query)
    finally:
        runtime.generate_partial_draft_rounds_from_cache = orig_draft
        runtime._keep_positions_for_chunk = orig_keep
        runtime._keep_positions_per_layer_per_head_for_chunk = orig_keep_ph
        runtime.query_attention_token_scores = orig_tok_scores
        runtime._forward_generation_block_replace = orig_fwd_replace
        runtime._selection_query_ids_with_score_target = orig_selection
    rec.update(
        sequences=list(result.sequences), selected_chunk_indices=list(result.selected_chunk_indices),
        chunk_scores={str(k): float(v) for k, v in result.chunk_scores.items()}, cache_tokens=result.cache_tokens,
        removed_tokens=result.removed_tokens, candidate_chunks=result.candidate_chunks, prefix_tokens=result.prefix_tokens,
        generation_blocks=result.generation_blocks,
        chunk_meta=[dict(chunk_index=m.chunk_index, original_tokens=m.original_tokens, kept_tokens=m.kept_tokens,
                         cache_start=m.cache_start, cache_end=m.cache_end, rope_start=m.rope_start, rope_end=m.rope_end)
                    for m in result.chunk_meta],
        block_states_before_each_forward=steps,
    )
    return rec


def cross_check_vendored_dream(reference_root: str, ckpt: str) -> float:
    """Max |logit| difference between the contract model and the Dream model the reference vendors
    (prefilling_dllm_eval/model_cache/dream/model_dream.py) on a plain full-attention forward."""
    eval_dir = os.path.join(reference_root, "prefilling_dllm_eval")
    if eval_dir not in sys.path:
        sys.path.insert(0, eval_dir)
    from fastdllm_v1_model import _ensure_default_rope_init

    _ensure_default_rope_init()
    from model_cache.dream.configuration_dream import DreamConfig as VendoredConfig
    from model_cache.dream.model_dream import DreamModel as VendoredDream
    from safetensors.torch import load_file

    from oracle.contract_model.model.modeling_dream import DreamModel

    vend = VendoredDream(VendoredConfig(**{k: v for k, v in TOY.items()}))
    state = load_file(os.path.join(ckpt, "model.safetensors"))
    vend.load_state_dict(state, strict=False)
    vend = vend.float().eval()
    mine = DreamModel.from_pretrained(ckpt).eval()
    ids = torch.randint(3, 1023, (1, 77), generator=torch.Generator().manual_seed(5))
    with torch.no_grad():
        a = vend(ids, attention_mask=None, position_ids=torch.arange(77).unsqueeze(0)).logits
        b = mine(ids, attention_mask="full", position_ids=torch.arange(77).unsqueeze(0)).logits
    return float((a - b).abs().max())


VARIANTS = {
    "readme_full_prompt_mask": dict(README_FLAGS),
    "chunk_query_reuse": dict(README_FLAGS, cache_build_mode="chunk_query", chunk_position_mode="reuse",
                              query_position_mode="after_reused_window"),
    "evict_global_cap128": dict(README_FLAGS, token_capacity=128),
    "evict_per_head_cap128_chunk_query": dict(README_FLAGS, token_capacity=128, token_eviction_granularity="per_head",
                                              cache_build_mode="chunk_query", chunk_position_mode="reuse",
                                              query_position_mode="after_reused_window"),
    "two_blocks": dict(README_FLAGS, max_new_tokens=64),
    "evict_per_head_cap128_full_prompt_two_blocks": dict(README_FLAGS, token_capacity=128, max_new_tokens=64,
                                                         token_eviction_granularity="per_head"),
    "full_prompt_query": dict(README_FLAGS, cache_build_mode="full_prompt_query"),
    # the config dataclass's own draft defaults: no partial rounds -> a full confidence-threshold draft of 16 tokens,
    # every query + draft position is a label
    "draft_dataclass_defaults": dict(README_FLAGS, score_draft_partial_rounds=None, score_draft_tokens=16),
    "draft_partial_steps": dict(README_FLAGS, score_draft_partial_rounds=None, score_draft_partial_steps=2),
    "draft_fixed_steps": dict(README_FLAGS, score_draft_partial_rounds=None, score_draft_fixed_steps=True, score_draft_steps=2),
}

# head_dim-128 toy: the README flow, and the sharded flow's flags (independent chunks, global eviction, two blocks)
VARIANTS128 = {
    "readme_full_prompt_mask": dict(README_FLAGS),
    "chunk_query_evict_global_cap128_two_blocks": dict(README_FLAGS, cache_build_mode="chunk_query", chunk_position_mode="reuse",
                                                       query_position_mode="after_reused_window", token_capacity=128,
                                                       max_new_tokens=64),
    "evict_per_head_cap128_full_prompt": dict(README_FLAGS, token_capacity=128, token_eviction_granularity="per_head"),
}

# flags off the README path (fp32 toy): score context / mask / mode, pooling and reductions of the token scores, score direction,
# deterministic sampler options (top-k / top-p at temperature 0, margin and entropy confidence with fixed-step diffusion)
_CHUNK_QUERY = dict(cache_build_mode="chunk_query", chunk_position_mode="reuse", query_position_mode="after_reused_window")
FLAG_VARIANTS = {
    "score_joint_chunks_target_last": dict(README_FLAGS, score_context_mode="joint_chunks_target_last"),
    "score_mask_query_to_chunk": dict(README_FLAGS, score_attention_mask="query_to_chunk"),
    "score_mask_full": dict(README_FLAGS, score_attention_mask="full"),
    "score_mode_self_information_window16": dict(README_FLAGS, score_mode="self_information", score_query_window=16),
    "score_mode_next_block_logits": dict(README_FLAGS, score_mode="next_block_logits"),
    "score_mode_attention": dict(README_FLAGS, score_mode="attention"),
    "score_mode_per_chunk_draft": dict(README_FLAGS, score_mode="per_chunk_draft_self_information"),
    "evict_avgpool_head_max_layer_sum": dict(README_FLAGS, token_capacity=128, token_score_pooling="avgpool", token_score_head_reduce="max",
                                             token_score_layer_reduce="sum"),
    "evict_nopool_head_mean_layer_max_keep_low": dict(README_FLAGS, token_capacity=128, token_score_pooling="none",
                                                      token_score_head_reduce="mean", token_score_layer_reduce="max", token_score_keep="low"),
    "evict_per_head_avgpool_chunk_query": dict(README_FLAGS, token_capacity=128, token_eviction_granularity="per_head",
                                               token_score_pooling="avgpool", **_CHUNK_QUERY),
    "evict_bidirectional_full_mask": dict(README_FLAGS, token_capacity=128, token_score_direction="bidirectional", token_attention_mask="full"),
    "evict_query_to_chunk_mask_chunk_query": dict(README_FLAGS, token_capacity=128, token_attention_mask="query_to_chunk", **_CHUNK_QUERY),
    "evict_use_generated_query": dict(README_FLAGS, token_capacity=128, token_score_use_generated=True),
    "sample_top_k_top_p_greedy": dict(README_FLAGS, top_k=8, top_p=0.7),
    # temperature > 0 draws from a categorical; with one candidate left per slot the draw is deterministic, every slot has
    # confidence 1 and a block fills in one step. Scored without a draft: WHICH of several slots of confidence exactly 1 a
    # draft round takes is torch.topk's unspecified choice among ties, and later rounds depend on it
    "sample_temperature_top_k_1": dict(README_FLAGS, score_mode="self_information", temperature=0.7, top_k=1),
    "alg_topk_margin": dict(README_FLAGS, alg="topk_margin", diffusion_steps=8),
    # YaRN context extension: inverse frequencies blended between extrapolation and interpolation, cos / sin scaled
    "rope_yarn_factor_4": dict(README_FLAGS, rope_scale_factor=4.0),
    "alg_entropy": dict(README_FLAGS, alg="entropy", diffusion_steps=8),
}


def record_drafts_on_cache(runtime, context, query) -> dict:
    """The two partial drafts of the reference class on top of an EXISTING cache (fastdllm_parallelcomp.py:2512-2676): the cache of the
    independently prefilled selected chunks (build_prefill_cache), the query forwarded against it, then the draft block."""
    cache, positions, _ = runtime.build_prefill_cache(prefix_ids=runtime.bos_ids(), context_ids=context, query_ids=query)
    start = max(positions) + 1
    rounds_ids, rounds_mask = runtime.generate_partial_draft_rounds_from_cache(
        past_key_values=cache, cache_positions=positions, query_ids=query, query_rope_start=start, max_new_tokens=6, partial_rounds=3)
    steps_ids, steps_filled = runtime.generate_partial_draft_from_cache(
        past_key_values=cache, cache_positions=positions, query_ids=query, query_rope_start=start, max_new_tokens=6, partial_steps=4)
    alone_ids, alone_mask = runtime.generate_partial_draft_rounds_from_cache(
        past_key_values=None, cache_positions=[], query_ids=query, query_rope_start=start, max_new_tokens=6, partial_rounds=3)
    return dict(cache_tokens=len(positions), query_rope_start=int(start), rounds=dict(ids=[int(t) for t in rounds_ids], mask=[bool(m) for m in rounds_mask]),
                steps=dict(ids=[int(t) for t in steps_ids], filled=int(steps_filled)),
                without_cache=dict(ids=[int(t) for t in alone_ids], mask=[bool(m) for m in alone_mask]))


DRAFT_ON_CACHE_VARIANTS = {
    "chunk_query_reuse": dict(README_FLAGS, cache_build_mode="chunk_query", chunk_position_mode="reuse", query_position_mode="after_reused_window"),
    "chunk_query_evict_global_cap128": dict(README_FLAGS, cache_build_mode="chunk_query", chunk_position_mode="reuse",
                                            query_position_mode="after_reused_window", token_capacity=128),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PDLLM_REFERENCE_ROOT"), required="PDLLM_REFERENCE_ROOT" not in os.environ,
                    help="root of the reference checkout (or set PDLLM_REFERENCE_ROOT)")
    ap.add_argument("--out", default=os.path.join(HERE, "toy_reference.json"))
    ap.add_argument("--out128", default=os.path.join(HERE, "toy128_reference.json"))
    ap.add_argument("--out-flags", default=os.path.join(HERE, "toy_flags_reference.json"))
    ap.add_argument("--out-drafts", default=os.path.join(HERE, "toy_draft_on_cache_reference.json"))
    ap.add_argument("--only", choices=["toy", "toy128", "flags", "drafts"], default=None)
    args = ap.parse_args()
    torch.manual_seed(0)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    with tempfile.TemporaryDirectory() as tmp:
        if args.only in (None, "toy"):
            context, query = toy_inputs()
            golden = {"config": dict(TOY), "flags": dict(README_FLAGS), "context_seed": 0, "runs": {}}
            ckpt = os.path.join(tmp, "ckpt_toy")
            write_toy_checkpoint(ckpt)
            try:
                golden["vendored_dream_max_abs_logit_diff"] = cross_check_vendored_dream(args.reference, ckpt)
            except Exception as exc:  # the vendored model depends on the installed transformers version
                golden["vendored_dream_max_abs_logit_diff"] = None
                golden["vendored_dream_error"] = f"{type(exc).__name__}: {exc}"
            for name, flags in VARIANTS.items():
                _, runtime = load_reference(args.reference, ckpt, **flags)
                golden["runs"][name] = dict(flags=flags, **record_run(runtime, context, query))
                print(name, golden["runs"][name]["selected_chunk_indices"], golden["runs"][name]["sequences"][:8])
            with open(args.out, "w") as handle:
                json.dump(golden, handle)
            print("wrote", args.out, os.path.getsize(args.out), "bytes")
        if args.only in (None, "flags"):
            context, query = toy_inputs()
            golden = {"config": dict(TOY), "flags": dict(README_FLAGS), "context_seed": 0, "runs": {}}
            ckpt = os.path.join(tmp, "ckpt_toy_flags")
            write_toy_checkpoint(ckpt)
            for name, flags in FLAG_VARIANTS.items():
                _, runtime = load_reference(args.reference, ckpt, **flags)
                golden["runs"][name] = dict(flags=flags, **record_run(runtime, context, query))
                print(name, golden["runs"][name]["selected_chunk_indices"], golden["runs"][name]["sequences"][:8], flush=True)
            with open(args.out_flags, "w") as handle:
                json.dump(golden, handle)
            print("wrote", args.out_flags, os.path.getsize(args.out_flags), "bytes")
        if args.only in (None, "drafts"):
            context, query = toy_inputs()
            golden = {"config": dict(TOY), "context_seed": 0, "runs": {}}
            ckpt = os.path.join(tmp, "ckpt_toy_drafts")
            write_toy_checkpoint(ckpt)
            for name, flags in DRAFT_ON_CACHE_VARIANTS.items():
                _, runtime = load_reference(args.reference, ckpt, **flags)
                golden["runs"][name] = dict(flags=flags, **record_drafts_on_cache(runtime, context, query))
                print(name, golden["runs"][name]["rounds"], golden["runs"][name]["steps"], golden["runs"][name]["without_cache"], flush=True)
            with open(args.out_drafts, "w") as handle:
                json.dump(golden, handle)
            print("wrote", args.out_drafts, os.path.getsize(args.out_drafts), "bytes")
        if args.only in (None, "toy128"):
            context, query = toy_inputs(vocab=TOY128["vocab_size"])
            golden = {"config": dict(TOY128), "flags": dict(README_FLAGS), "context_seed": 0, "runs": {}}
            ckpt = os.path.join(tmp, "ckpt_toy128")
            write_toy_checkpoint(ckpt, config=TOY128)
            for dtype in ("float32", "bfloat16"):
                for name, flags in VARIANTS128.items():
                    _, runtime = load_reference(args.reference, ckpt, dtype=dtype, **flags)
                    key = f"{name}/{dtype}"
                    golden["runs"][key] = dict(flags=flags, dtype=dtype, **record_run(runtime, context, query))
                    print(key, golden["runs"][key]["selected_chunk_indices"], golden["runs"][key]["sequences"][:8])
            with open(args.out128, "w") as handle:
                json.dump(golden, handle)
            print("wrote", args.out128, os.path.getsize(args.out128), "bytes")


if __name__ == "__main__":
    main()
