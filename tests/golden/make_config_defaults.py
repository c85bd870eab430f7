"""Writes tests/golden/config_defaults.json: field names and default values of the reference's
FastDLLMParallelCompConfig, FastDLLMChunkMeta and FastDLLMParallelCompResult dataclasses
(prefilling_dllm_eval/fastdllm_parallelcomp.py), read by importing the unmodified reference module on CPU.

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
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "prefilling_dllm_eval"))
    import fastdllm_parallelcomp as ref

    data = {name: describe(getattr(ref, name)) for name in ("FastDLLMParallelCompConfig", "FastDLLMChunkMeta", "FastDLLMParallelCompResult")}
    with open(os.path.join(HERE, "config_defaults.json"), "w") as handle:
        json.dump(data, handle, indent=1, sort_keys=True)
    print({k: len(v) for k, v in data.items()})


if __name__ == "__main__":
    main()
