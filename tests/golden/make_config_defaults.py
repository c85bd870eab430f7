"""Writes tests/golden/config_defaults.json: field names and default values of the reference's
FastDLLMParallelCompConfig, FastDLLMChunkMeta and FastDLLMParallelCompResult dataclasses and the signatures of the
public methods of FastDLLMParallelComp (prefilling_dllm_eval/fastdllm_parallelcomp.py), read by importing the unmodified reference module on CPU.

    python tests/golden/make_config_defaults.py [--reference /path/to/reference]
"""

import argparse
import dataclasses
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def describe(cls):
    out = {}
    for f in dataclasses.fields(cls):
        if f.default is not dataclasses.MISSING:
            default = f.default
        elif f.default_factory is not dataclasses.MISSING:  # type: ignore[misc]
            default = f.default_factory()                    # type: ignore[misc]
        else:
            default = "<required>"
        out[f.name] = default if isinstance(default, (int, float, str, bool, type(None), list, dict)) else repr(default)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PDLLM_REFERENCE_ROOT"), required="PDLLM_REFERENCE_ROOT" not in os.environ,
                    help="root of the reference checkout (or set PDLLM_REFERENCE_ROOT)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "prefilling_dllm_eval"))
    import fastdllm_parallelcomp as ref

    import inspect

    data = {name: describe(getattr(ref, name)) for name in ("FastDLLMParallelCompConfig", "FastDLLMChunkMeta", "FastDLLMParallelCompResult")}
    methods = {}
    for name in ("generate", "generate_from_text_parts", "generate_from_cache", "generate_full_prompt_mask", "build_prefill_cache",
                 "select_chunks", "score_chunks_self_information_batched", "generate_partial_draft_rounds_from_cache",
                 "encode_fragment", "bos_ids"):
        params = list(inspect.signature(getattr(ref.FastDLLMParallelComp, name)).parameters.values())[1:]
        methods[name] = [[p.name, p.kind == p.KEYWORD_ONLY,
                          "<required>" if p.default is inspect.Parameter.empty else (p.default if isinstance(p.default, (int, float, str, bool, type(None))) else repr(p.default))]
                         for p in params]
    data["FastDLLMParallelComp.methods"] = methods
    data["module_functions"] = {name: [p.name for p in inspect.signature(getattr(ref, name)).parameters.values()]
                                for name in ("split_token_chunks", "load_fastdllm_parallelcomp")}
    with open(os.path.join(HERE, "config_defaults.json"), "w") as handle:
        json.dump(data, handle, indent=1, sort_keys=True)
    print({k: len(v) for k, v in data.items()})


if __name__ == "__main__":
    main()
