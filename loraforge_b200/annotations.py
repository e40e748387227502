"""Stability metadata for public experimental APIs.

Same contract as the reference's ``loraforge.annotations`` (src/loraforge/annotations.py:16-86):
decorated callables carry ``__experimental_api__`` (reason, since, stability
"alpha") and a docstring note; with ``warn=True`` a synchronous function warns
once per process.  Numerical operators are returned unwrapped.
"""

from __future__ import annotations

import inspect
import os
import threading
import warnings
from dataclasses import dataclass
from functools import wraps


class ExperimentalAPIWarning(UserWarning):
    """The decorated API is public but carries no compatibility guarantee yet."""


@dataclass(frozen=True)
class ExperimentalInfo:
    reason: str
    since: str
    stability: str = "alpha"


def ExperimentalAPI(*, reason: str, since: str = "0.1.0.dev0", warn: bool = False):
    """Attach alpha-stability metadata; optionally warn once per process."""
    if not isinstance(reason, str) or not reason.strip():
        raise ValueError("reason must be a nonempty description")
    if not isinstance(since, str) or not since.strip():
        raise ValueError("since must be a nonempty version string")
    if type(warn) is not bool:
        raise TypeError("warn must be a bool")
    info = ExperimentalInfo(reason=reason, since=since)

    def decorate(obj):
        if not callable(obj):
            raise TypeError("ExperimentalAPI requires a callable")
        plain_function = inspect.isfunction(obj) and not (
            inspect.iscoroutinefunction(obj)
            or inspect.isgeneratorfunction(obj)
            or inspect.isasyncgenfunction(obj)
        )
        if warn and not plain_function:
            raise TypeError("warn=True requires a synchronous non-generator function")
        obj.__experimental_api__ = info
        obj.__doc__ = (obj.__doc__ or "") + (
            f"\n\nExperimental API (alpha, since {since}). {reason} "
            "API compatibility is not guaranteed."
        )
        if not warn:
            return obj
        seen: set[int] = set()
        lock = threading.Lock()

        @wraps(obj)
        def wrapper(*args, **kwargs):
            pid = os.getpid()
            if pid not in seen:
                with lock:
                    if pid not in seen:
                        seen.add(pid)
                        warnings.warn(
                            f"{obj.__module__}.{obj.__qualname__} is experimental. {reason}",
                            ExperimentalAPIWarning,
                            stacklevel=2,
                        )
            return obj(*args, **kwargs)

        return wrapper

    return decorate
