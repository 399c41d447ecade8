"""Import shim for the package directory `verum-bespoke-singularity_b200/`.

The directory name contains hyphens, which Python cannot import by name;
`import vbs_b200` from the repository root loads its __init__.py under this
module name instead.
"""
import importlib.util as _ilu
import pathlib as _pl
import sys as _sys

_DIR = _pl.Path(__file__).resolve().parent / "verum-bespoke-singularity_b200"
_spec = _ilu.spec_from_file_location(__name__, _DIR / "__init__.py", submodule_search_locations=[str(_DIR)])
_mod = _ilu.module_from_spec(_spec)
_sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
