"""tpcuda: B200 CUDA backend for the torch-pyodide tensor-op hot path.

``CudaRuntime`` mirrors the reference runtime's op surface over libtpcuda.so;
``shim.install(runtime)`` makes the reference ``torch`` package use it.
"""
from .runtime import CudaRuntime  # noqa: F401
from . import shim  # noqa: F401

__all__ = ["CudaRuntime", "shim"]
