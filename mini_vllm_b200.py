"""Import shim: ``import mini_vllm_b200`` loads the package that lives in the
directory ``mini-vllm-continuous-batching-lab_b200/`` next to this file.

The directory name carries hyphens, which Python's import statement cannot
spell, so this module replaces itself in ``sys.modules`` with the package
(its ``__path__`` set to that directory) and submodule imports such as
``import mini_vllm_b200.attention`` then resolve inside it.
"""

import importlib.util as _ilu
import os as _os
import sys as _sys

_PKG_DIR = _os.path.join(
    _os.path.dirname(_os.path.abspath(__file__)), "mini-vllm-continuous-batching-lab_b200"
)
_spec = _ilu.spec_from_file_location(
    __name__, _os.path.join(_PKG_DIR, "__init__.py"), submodule_search_locations=[_PKG_DIR]
)
_pkg = _ilu.module_from_spec(_spec)
_sys.modules[__name__] = _pkg
_spec.loader.exec_module(_pkg)
