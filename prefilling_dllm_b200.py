"""Import alias: `import prefilling_dllm_b200` loads the package kept in the `prefilling-dllm_b200/` directory
(a directory name with a hyphen cannot be imported directly)."""

import importlib.util as _util
import os as _os
import sys as _sys

_pkg_dir = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "prefilling-dllm_b200")
_spec = _util.spec_from_file_location(
    __name__, _os.path.join(_pkg_dir, "__init__.py"), submodule_search_locations=[_pkg_dir]
)
_module = _util.module_from_spec(_spec)
_sys.modules[__name__] = _module
_spec.loader.exec_module(_module)
