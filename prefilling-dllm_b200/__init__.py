"""B200-native kernels and host logic for the Prefilling-dLLM long-context hot path.

Import name: `prefilling_dllm_b200` (the alias module at the repository root maps it onto this directory).
`ops` is the reference-compatible op table over the C-ABI library; nothing here falls back to CPU.
"""

from . import _lib, ops  # noqa: F401

__all__ = ["_lib", "ops"]
