"""Drop-in boundary: stand-ins for the two Pyodide modules the reference imports.

The reference ``torch`` package reaches its runtime through exactly two names
(python/torch/_runtime.py:15-39):

  * ``from js import globalThis`` and ``getattr(globalThis,
    "__torch_pyodide_runtime__")`` to find the runtime object;
  * ``from pyodide.ffi import can_run_sync, run_sync`` to await each JS
    promise synchronously.

``install(runtime)`` registers a ``js`` module whose ``globalThis`` carries the
given runtime, and a ``pyodide.ffi`` module whose ``run_sync`` is the identity
(every runtime method here returns its result directly, so there is nothing to
await) and whose ``can_run_sync`` is true.  The reference package then runs
unedited on top of the CUDA runtime.
"""
from __future__ import annotations

import sys
import types

RUNTIME_GLOBAL_KEY = "__torch_pyodide_runtime__"


class _GlobalThis:
    """Attribute bag standing in for the browser's ``globalThis``."""


def run_sync(value):
    return value


def can_run_sync() -> bool:
    return True


def install(runtime) -> None:
    """Expose ``runtime`` as ``globalThis.__torch_pyodide_runtime__``."""
    js = sys.modules.get("js")
    if js is None or not hasattr(js, "globalThis"):
        js = types.ModuleType("js")
        js.globalThis = _GlobalThis()
        sys.modules["js"] = js
    setattr(js.globalThis, RUNTIME_GLOBAL_KEY, runtime)

    pyodide = sys.modules.get("pyodide") or types.ModuleType("pyodide")
    ffi = types.ModuleType("pyodide.ffi")
    ffi.run_sync = run_sync
    ffi.can_run_sync = can_run_sync
    pyodide.ffi = ffi
    sys.modules["pyodide"] = pyodide
    sys.modules["pyodide.ffi"] = ffi


def uninstall() -> None:
    for name in ("js", "pyodide.ffi", "pyodide"):
        sys.modules.pop(name, None)
