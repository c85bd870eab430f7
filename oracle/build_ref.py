"""Stage the reference's own implementation of the path under oracle/_ref/ (git-ignored). TEST INFRASTRUCTURE ONLY.

The reference is pure Python: there is nothing to compile. Its files for this path are copied byte for byte from a
reference checkout into oracle/_ref/, which is kept out of the repository's history and only travels with a working copy
to a GPU machine, where the checkout itself does not exist:

  * prefilling_dllm_eval/fastdllm_parallelcomp.py + fastdllm_v1_model.py — the eval class, run UNMODIFIED on the host cores
    over oracle/contract_model as the CPU baseline of bench.py;
  * prefilling_dllm_engine/prefilling_dllm/layers/attention/ops/{prefix_prefill, chunked_prefill_decoding_unified_kernel,
    kv_cache_kernels, triton_eviction_scorer}.py — the reference's Triton kernels, which on a GPU machine pin the op-level
    oracle (tests/test_gpu_reference_kernels.py) and are the same-box baseline that bench.py times.

  * prefilling_dllm_engine/prefilling_dllm/ (the whole engine package, 0.7 MB) + prefilling_dllm_eval/model_cache/dream/
    configuration_dream.py — the reference's PD engine `FastDLLMDreamEngine`, which constructs CUDA state and therefore runs
    on a GPU machine only: tests/golden/make_engine_golden.py drives it there, unmodified, over the toy checkpoint and
    writes the fixture that pins oracle/engine_flow.py and the engine facade of this library.

    python oracle/build_ref.py --reference /path/to/reference        (or PDLLM_REFERENCE_ROOT)

`load_eval_module()` / `load_engine_ops()` import the staged files; they raise RefUnavailable when nothing was staged.
Nothing in the product package imports this module.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import shutil
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
EVAL_FILES = ["fastdllm_parallelcomp.py", "fastdllm_v1_model.py"]
OPS_DIR = os.path.join("prefilling_dllm_engine", "prefilling_dllm", "layers", "attention", "ops")
OPS_FILES = ["prefix_prefill.py", "chunked_prefill_decoding_unified_kernel.py", "kv_cache_kernels.py", "triton_eviction_scorer.py"]


class RefUnavailable(RuntimeError):
    pass


def stage(reference_root: str) -> str:
    """Copy the files listed above into oracle/_ref/{eval,ops}/. Returns the directory."""
    for sub, names, src_dir in (("eval", EVAL_FILES, os.path.join(reference_root, "prefilling_dllm_eval")),
                                ("ops", OPS_FILES, os.path.join(reference_root, OPS_DIR))):
        dst_dir = os.path.join(REF_DIR, sub)
        os.makedirs(dst_dir, exist_ok=True)
        for name in names:
            shutil.copyfile(os.path.join(src_dir, name), os.path.join(dst_dir, name))
    # the engine package as a tree, and the configuration class a Dream checkpoint names in its auto_map
    engine_dst = os.path.join(REF_DIR, "engine")
    if os.path.isdir(os.path.join(engine_dst, "prefilling_dllm")):
        shutil.rmtree(os.path.join(engine_dst, "prefilling_dllm"))
    shutil.copytree(os.path.join(reference_root, "prefilling_dllm_engine", "prefilling_dllm"), os.path.join(engine_dst, "prefilling_dllm"),
                    ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    shutil.copyfile(os.path.join(reference_root, "prefilling_dllm_eval", "model_cache", "dream", "configuration_dream.py"),
                    os.path.join(engine_dst, "configuration_dream.py"))
    return REF_DIR


def engine_staged() -> bool:
    return os.path.exists(os.path.join(REF_DIR, "engine", "prefilling_dllm", "fastdllm_engine.py"))


def load_reference_engine():
    """The reference's `prefilling_dllm.fastdllm_engine` module, imported from the staged package tree (GPU machine only: its
    model runner initialises CUDA and NCCL). `easydict` is served by oracle/shims when the image lacks it."""
    if not engine_staged():
        raise RefUnavailable("oracle/_ref/engine is empty: run oracle/build_ref.py where a reference checkout exists")
    for name in [n for n in sys.modules if n == "prefilling_dllm" or n.startswith("prefilling_dllm.")]:
        del sys.modules[name]           # stand-ins left by load_engine_ops()
    root = os.path.join(REF_DIR, "engine")
    if root not in sys.path:
        sys.path.insert(0, root)
    try:
        import easydict  # noqa: F401
    except ImportError:
        sys.path.append(os.path.join(HERE, "shims"))
    import prefilling_dllm.fastdllm_engine as module  # noqa: the staged, unmodified reference engine

    return module


def staged() -> bool:
    return all(os.path.exists(os.path.join(REF_DIR, "eval", n)) for n in EVAL_FILES) and \
        all(os.path.exists(os.path.join(REF_DIR, "ops", n)) for n in OPS_FILES)


def load_eval_module():
    """The reference's fastdllm_parallelcomp module, imported from the staged copy."""
    path = os.path.join(REF_DIR, "eval")
    if not os.path.exists(os.path.join(path, EVAL_FILES[0])):
        raise RefUnavailable("oracle/_ref/eval is empty: run oracle/build_ref.py where a reference checkout exists")
    if path not in sys.path:
        sys.path.insert(0, path)
    import fastdllm_parallelcomp  # noqa: the staged, unmodified reference module

    return fastdllm_parallelcomp


def _load(name: str, path: str):
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


def load_engine_ops():
    """Namespace with the reference's Triton entry points: context_attention_fwd, chunked_prefill_paged_decode,
    store_kvcache_unified_layout, store_kvcache_distinct_layout, load_kvcache (the undecorated function),
    query_to_chunk_attention_scores. Needs a GPU machine with triton (and vllm, which the reference imports for platform
    probing only; when vllm cannot be imported a stand-in with the few attributes the files read is used and
    `stubbed_vllm` is set). The engine package modules the op files import for type annotations only are stand-ins."""
    ops_dir = os.path.join(REF_DIR, "ops")
    if not os.path.exists(os.path.join(ops_dir, OPS_FILES[0])):
        raise RefUnavailable("oracle/_ref/ops is empty: run oracle/build_ref.py where a reference checkout exists")
    import torch

    stubbed = False
    try:
        import vllm.platforms  # noqa
        from vllm import _custom_ops  # noqa
    except Exception:  # any failure of the third-party import: the kernels themselves do not need it
        stubbed = True
        for name in [n for n in sys.modules if n == "vllm" or n.startswith("vllm.")]:
            del sys.modules[name]
        vllm = types.ModuleType("vllm")
        platforms = types.ModuleType("vllm.platforms")

        class _Platform:
            @staticmethod
            def is_rocm():
                return False

            @staticmethod
            def is_cuda():
                return True

            @staticmethod
            def fp8_dtype():
                return torch.float8_e4m3fn

            @staticmethod
            def has_device_capability(*a, **k):
                return True

        platforms.current_platform = _Platform()
        vllm.platforms = platforms
        vllm._custom_ops = types.ModuleType("vllm._custom_ops")
        sys.modules.update({"vllm": vllm, "vllm.platforms": platforms, "vllm._custom_ops": vllm._custom_ops})
    # engine modules that the op files import for annotations only
    pkg_names = ["prefilling_dllm", "prefilling_dllm.utils", "prefilling_dllm.utils.context", "prefilling_dllm.engine",
                 "prefilling_dllm.engine.sequence", "prefilling_dllm.layers", "prefilling_dllm.layers.attention",
                 "prefilling_dllm.layers.attention.ops"]
    for name in pkg_names:
        if name not in sys.modules:
            mod = types.ModuleType(name)
            mod.__path__ = []
            sys.modules[name] = mod
    sys.modules["prefilling_dllm.utils.context"].ContextForDiffusionLM = type("ContextForDiffusionLM", (), {})
    sys.modules["prefilling_dllm.engine.sequence"].SequenceForDiffusionLM = type("SequenceForDiffusionLM", (), {})
    base = "prefilling_dllm.layers.attention.ops."
    prefix = _load(base + "prefix_prefill", os.path.join(ops_dir, "prefix_prefill.py"))
    unified = _load(base + "chunked_prefill_decoding_unified_kernel", os.path.join(ops_dir, "chunked_prefill_decoding_unified_kernel.py"))
    kv = _load(base + "kv_cache_kernels", os.path.join(ops_dir, "kv_cache_kernels.py"))
    scorer = _load(base + "triton_eviction_scorer", os.path.join(ops_dir, "triton_eviction_scorer.py"))
    ns = types.SimpleNamespace(
        context_attention_fwd=prefix.context_attention_fwd, chunked_prefill_paged_decode=unified.chunked_prefill_paged_decode,
        store_kvcache_unified_layout=kv.store_kvcache_unified_layout, store_kvcache_distinct_layout=kv.store_kvcache_distinct_layout,
        # the reference decorates this host function with @triton.jit; its body is the plain function underneath
        load_kvcache=getattr(kv.load_kvcache, "fn", kv.load_kvcache),
        query_to_chunk_attention_scores=scorer.query_to_chunk_attention_scores, stubbed_vllm=stubbed)
    return ns


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PDLLM_REFERENCE_ROOT"), required="PDLLM_REFERENCE_ROOT" not in os.environ)
    args = ap.parse_args()
    print("staged the reference files under", stage(args.reference))


if __name__ == "__main__":
    main()
