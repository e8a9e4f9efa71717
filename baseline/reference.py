"""Import the reference package installed under ``baseline/_ref`` (test and
measurement infrastructure only; ``piper_offload_b200`` never imports it).

The reference declares Python >= 3.14, whose annotations are evaluated lazily.
On this interpreter (3.12) its modules are compiled with postponed
annotations (``from __future__ import annotations``), which is the only
difference to importing them normally; the sources are unmodified copies made
by ``baseline/install_reference.py``.
"""

from __future__ import annotations

import __future__
import importlib
import importlib.abc
import importlib.machinery
import sys
from pathlib import Path

REF_ROOT = Path(__file__).resolve().parent / "_ref"
_installed = False


def available() -> bool:
    return (REF_ROOT / "piper_offload" / "__init__.py").exists()


def _install_hook() -> None:
    global _installed
    if _installed:
        return

    class _Loader(importlib.machinery.SourceFileLoader):
        def source_to_code(self, data, path, *, _optimize=-1):  # noqa: ANN001
            return compile(data, path, "exec", flags=__future__.annotations.compiler_flag, dont_inherit=True,
                           optimize=_optimize)

    class _Finder(importlib.abc.MetaPathFinder):
        def find_spec(self, name, path, target=None):  # noqa: ANN001, ARG002
            if name != "piper_offload" and not name.startswith("piper_offload."):
                return None
            spec = importlib.machinery.PathFinder.find_spec(name, path or [str(REF_ROOT)])
            if spec and spec.origin and spec.origin.endswith(".py"):
                spec.loader = _Loader(name, spec.origin)
            return spec

    sys.meta_path.insert(0, _Finder())
    _installed = True


def load(module: str = "piper_offload"):
    """Import ``module`` (``piper_offload`` or one of its submodules) from the
    reference install; raises ImportError when it is absent."""
    if not available():
        raise ImportError(f"reference not installed under {REF_ROOT} (run baseline/install_reference.py)")
    _install_hook()
    return importlib.import_module(module)
