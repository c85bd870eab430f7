"""Stand-in for the Fast-dLLM v1 `model` package (NVlabs/Fast-dLLM, v1/dream/model), which the reference loads
by directory (prefilling_dllm_eval/fastdllm_parallelcomp.py:411-437) and does not vendor. TEST INFRASTRUCTURE."""
