"""Writes tests/golden/engine_api.json: dataclass fields and public method signatures of the reference engine
(prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py), read from its source with `ast` (the module itself
initialises CUDA and cannot be imported on a CPU box).

    python tests/golden/make_engine_api.py [--reference /path/to/reference]
"""

import argparse
import ast
import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))
METHODS = ["__init__", "prefill_to_pd_record", "decode_from_pd_record", "release_pd_record", "snapshot_pd_record_kv",
           "make_pd_record_from_kv_snapshot", "make_pd_record_from_remote_engine", "generate_token_ids_pd_split", "generate_token_ids",
           "generate", "select_chunks_by_engine", "score_chunk_self_information_engine", "generate_partial_draft_rounds_for_selection",
           "compute_prompt_keep_indices_per_layer_per_head", "generate_token_ids_from_chunk_local_kv", "close"]


def literal(node):
    try:
        return ast.literal_eval(node)
    except Exception:
        return ast.unparse(node)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PDLLM_REFERENCE_ROOT"), required="PDLLM_REFERENCE_ROOT" not in os.environ,
                    help="root of the reference checkout (or set PDLLM_REFERENCE_ROOT)")
    args = ap.parse_args()
    path = os.path.join(args.reference, "prefilling_dllm_engine", "prefilling_dllm", "fastdllm_engine.py")
    tree = ast.parse(open(path).read())
    out = {"dataclasses": {}, "methods": {}}
    for node in tree.body:
        if isinstance(node, ast.ClassDef) and node.name in {"FastDLLMEngineOutput", "DreamPrefillRecord", "DreamKVSnapshot"}:
            fields = []
            for item in node.body:
                if isinstance(item, ast.AnnAssign):
                    fields.append([item.target.id, "<required>" if item.value is None else literal(item.value)])
            out["dataclasses"][node.name] = fields
        if isinstance(node, ast.ClassDef) and node.name == "FastDLLMDreamEngine":
            for item in node.body:
                if isinstance(item, ast.FunctionDef) and item.name in METHODS:
                    a = item.args
                    pos = [x.arg for x in a.args][1:]
                    pos_defaults = [literal(d) for d in a.defaults]
                    kwonly = [[x.arg, "<required>" if d is None else literal(d)] for x, d in zip(a.kwonlyargs, a.kw_defaults)]
                    out["methods"][item.name] = {"positional": pos, "positional_defaults": pos_defaults, "keyword_only": kwonly}
    with open(os.path.join(HERE, "engine_api.json"), "w") as handle:
        json.dump(out, handle, indent=1, sort_keys=True)
    print(sorted(out["methods"]), {k: len(v) for k, v in out["dataclasses"].items()})


if __name__ == "__main__":
    main()
