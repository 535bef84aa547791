"""Log level of the library's own messages, numbered as in nvdiffrast (diffrast log.py:1-38)."""

from __future__ import annotations

import operator
import warnings

INFO, WARNING, ERROR, FATAL = range(4)

_level = WARNING


def get_log_level() -> int:
    """Current log level: 0 info, 1 warning (default), 2 error, 3 fatal."""
    return _level


def set_log_level(level: int) -> None:
    """Set the lowest level reported; warnings show at 0 and 1, errors always raise."""
    global _level
    try:
        value = operator.index(level)
    except TypeError:
        raise TypeError(f"level must be an int from 0 to 3, got {level!r}.") from None
    if not INFO <= value <= FATAL:
        raise ValueError(f"level must be an int from 0 to 3, got {level!r}.")
    _level = value


def warn(message: str, stacklevel: int = 1) -> None:
    """``UserWarning`` attributed to the caller unless the level silences warnings."""
    if _level <= WARNING:
        warnings.warn(message, stacklevel=stacklevel + 1)
