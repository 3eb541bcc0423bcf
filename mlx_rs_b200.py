"""Import shim for the package in ``mlx-rs_b200/``.

The package directory carries the project's name, which is not a Python identifier;
``import mlx_rs_b200`` loads it from there under this name.
"""
import importlib.util as _ilu
import os as _os
import sys as _sys

_ROOT = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "mlx-rs_b200")
_spec = _ilu.spec_from_file_location(__name__, _os.path.join(_ROOT, "__init__.py"),
                                     submodule_search_locations=[_ROOT])
_mod = _ilu.module_from_spec(_spec)
_sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
