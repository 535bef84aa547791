"""Run code written for nvdiffrast (or diffrast) on diffrast_b200 without editing it
(diffrast ``compat.py``).

:func:`install_as_nvdiffrast` makes ``import nvdiffrast.torch as dr`` resolve to this package;
:func:`install_as_diffrast` does the same for ``import diffrast``, so switching from diffrast is a
one-line change. Each registers two ``sys.modules`` entries (the package and its ``.torch``
module) and can be undone. Without ``force=True`` an alias refuses to shadow a real package of
that name, imported or merely installed.
"""

from __future__ import annotations

import importlib
import importlib.util
import sys
from types import ModuleType

from diffrast_b200 import log


class _ModuleAlias:
    """The pair of ``sys.modules`` entries that make ``name`` and ``name.torch`` this package."""

    def __init__(self, name: str) -> None:
        self.name = name
        self.saved: dict[str, ModuleType] = {}  # real modules set aside by a forced install

    def targets(self) -> dict[str, ModuleType]:
        return {
            self.name: importlib.import_module("diffrast_b200"),
            f"{self.name}.torch": importlib.import_module("diffrast_b200.torch"),
        }

    def install(self, force: bool) -> None:
        targets = self.targets()
        # Entries that hold something other than this package (a real, imported package).
        occupied = {key: sys.modules[key] for key, ours in targets.items()
                    if sys.modules.get(key, ours) is not ours}
        active = all(sys.modules.get(key) is ours for key, ours in targets.items())
        if active:
            return
        if not force:
            self._refuse(occupied)
        if occupied:
            log.warn(
                f"Replacing the imported {self.name} with diffrast_b200; modules that imported "
                "it earlier keep using it.",
                stacklevel=3,
            )
            self.saved.update(occupied)
        sys.modules.update(targets)

    def _refuse(self, occupied: dict[str, ModuleType]) -> None:
        if occupied:
            first = next(key for key in self.targets() if key in occupied)
            raise RuntimeError(
                f"{first} is already imported; pass force=True to replace it with diffrast_b200."
            )
        if self.name not in sys.modules and _findable(self.name):
            raise RuntimeError(
                f"A {self.name} package is installed; pass force=True to use diffrast_b200 in its "
                "place."
            )

    def uninstall(self) -> None:
        for key, ours in self.targets().items():
            displaced = self.saved.pop(key, None)
            if sys.modules.get(key) is not ours:
                continue
            if displaced is None:
                del sys.modules[key]
            else:
                sys.modules[key] = displaced


def _findable(name: str) -> bool:
    """Whether an importable package ``name`` exists (not counting a ``sys.modules`` entry)."""
    try:
        return importlib.util.find_spec(name) is not None
    except (ImportError, ValueError):
        return False


_ALIASES = {name: _ModuleAlias(name) for name in ("nvdiffrast", "diffrast")}


def install_as_nvdiffrast(force: bool = False) -> None:
    """Make ``import nvdiffrast.torch as dr`` resolve to diffrast_b200 in this process.

    Call it before importing code that uses nvdiffrast; modules that imported the real package
    earlier keep it. A second call does nothing.

    Args:
        force: Take the place of a real nvdiffrast that is installed or already imported (with a
            warning in the second case) instead of raising ``RuntimeError``.
    """
    _ALIASES["nvdiffrast"].install(force)


def uninstall_as_nvdiffrast() -> None:
    """Undo :func:`install_as_nvdiffrast`, putting back any modules it replaced."""
    _ALIASES["nvdiffrast"].uninstall()


def install_as_diffrast(force: bool = False) -> None:
    """Make ``import diffrast`` (and ``diffrast.torch``) resolve to diffrast_b200 in this
    process; ``force`` as for :func:`install_as_nvdiffrast`."""
    _ALIASES["diffrast"].install(force)


def uninstall_as_diffrast() -> None:
    """Undo :func:`install_as_diffrast`, putting back any modules it replaced."""
    _ALIASES["diffrast"].uninstall()
