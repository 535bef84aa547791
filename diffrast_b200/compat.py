"""Run code written for nvdiffrast (or diffrast) on diffrast_b200 without editing it.

:func:`install_as_nvdiffrast` registers this package under the module names ``nvdiffrast`` and
``nvdiffrast.torch`` (diffrast compat.py:15-74); :func:`install_as_diffrast` does the same for
``diffrast`` and ``diffrast.torch``, so switching from diffrast is a one-line change.
"""

from __future__ import annotations

import importlib
import importlib.util
import sys
from types import ModuleType

from diffrast_b200 import log

_displaced: dict[str, ModuleType] = {}


def _modules(name: str) -> dict[str, ModuleType]:
    return {
        name: importlib.import_module("diffrast_b200"),
        f"{name}.torch": importlib.import_module("diffrast_b200.torch"),
    }


def _install(name: str, force: bool) -> None:
    ours = _modules(name)
    current = {n: sys.modules.get(n) for n in ours}
    if all(current[n] is m for n, m in ours.items()):
        return
    imported = [n for n, m in ours.items() if current[n] not in (None, m)]
    if not force:
        if imported:
            raise RuntimeError(
                f"{imported[0]} is already imported; pass force=True to replace it with diffrast_b200."
            )
        if current[name] is None and _is_installed(name):
            raise RuntimeError(
                f"A {name} package is installed; pass force=True to use diffrast_b200 in its place."
            )
    if imported:
        log.warn(
            f"Replacing the imported {name} with diffrast_b200; modules that imported it "
            "earlier keep using it.",
            stacklevel=3,
        )
    for n, m in ours.items():
        if n in imported:
            _displaced[n] = current[n]
        sys.modules[n] = m


def _uninstall(name: str) -> None:
    for n, m in _modules(name).items():
        previous = _displaced.pop(n, None)
        if sys.modules.get(n) is m:
            del sys.modules[n]
            if previous is not None:
                sys.modules[n] = previous


def install_as_nvdiffrast(force: bool = False) -> None:
    """Make ``import nvdiffrast.torch as dr`` resolve to diffrast_b200 in this process."""
    _install("nvdiffrast", force)


def uninstall_as_nvdiffrast() -> None:
    """Undo :func:`install_as_nvdiffrast`, restoring any modules it replaced."""
    _uninstall("nvdiffrast")


def install_as_diffrast(force: bool = False) -> None:
    """Make ``import diffrast`` resolve to diffrast_b200 in this process."""
    _install("diffrast", force)


def uninstall_as_diffrast() -> None:
    """Undo :func:`install_as_diffrast`."""
    _uninstall("diffrast")


def _is_installed(name: str) -> bool:
    try:
        return importlib.util.find_spec(name) is not None
    except (ImportError, ValueError):
        return False
