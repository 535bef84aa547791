"""Verbosity of the library's own messages, with nvdiffrast's numbering (diffrast ``log.py``):
0 info, 1 warning (the default), 2 error, 3 fatal. Messages at warning level are issued as
``UserWarning`` while the level is at most 1; errors are exceptions and are raised whatever the
level is.
"""

from __future__ import annotations

import warnings

LEVELS = ("info", "warning", "error", "fatal")
INFO, WARNING, ERROR, FATAL = (LEVELS.index(name) for name in LEVELS)


class _Verbosity:
    """Holder of the process-wide level (one object, so no ``global`` statements are needed)."""

    value = WARNING


def _parse_level(level) -> int:
    message = f"level must be an int from 0 to 3, got {level!r}."
    index = getattr(type(level), "__index__", None)
    if index is None:
        raise TypeError(message)
    value = index(level)
    if value not in range(len(LEVELS)):
        raise ValueError(message)
    return value


def get_log_level() -> int:
    """The lowest level of message reported: 0 info, 1 warning, 2 error, 3 fatal."""
    return _Verbosity.value


def set_log_level(level: int) -> None:
    """Report messages from ``level`` (an int from 0 to 3) upwards."""
    _Verbosity.value = _parse_level(level)


def warn(message: str, stacklevel: int = 1) -> None:
    """Issue ``message`` as a ``UserWarning`` pointing at the caller's caller (``stacklevel``
    counts from the function that calls this one), unless the level is above warning."""
    if _Verbosity.value > WARNING:
        return
    warnings.warn(message, UserWarning, stacklevel=stacklevel + 1)
