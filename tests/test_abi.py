"""The C-ABI library: builds, loads without a GPU, exports every symbol that
include/tpcuda.h declares, and the ctypes binding covers them all."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tpcuda.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"TP_API\s+[\w\s\*]+?\b(tpk?_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from tpcuda import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from tpcuda.build import build
        build()
    return ctypes.CDLL(_lib.LIB_PATH)


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert len(syms) > 50
    assert "tp_adamw_step_multi" in syms and "tp_to_host" in syms


def test_every_declared_symbol_is_exported(lib):
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_ctypes_binding_covers_header():
    from tpcuda import _lib
    missing = [s for s in declared_symbols() if s not in _lib.SIGNATURES]
    extra = [s for s in _lib.SIGNATURES if s not in declared_symbols()]
    assert not missing and not extra, (missing, extra)


def test_no_device_reports_unavailable(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert lib.tp_is_available() == 0
    lib.tp_init.argtypes = [ctypes.c_int]
    assert lib.tp_init(0) != 0  # an error status, not a crash or a CPU fallback
    lib.tp_last_error.restype = ctypes.c_char_p
    assert b"CUDA" in lib.tp_last_error()


def test_tuning_switches_check_arguments_without_a_device(lib):
    """The tuning setters only record a value: they work with no GPU, refuse
    values outside their documented ranges with a message, and are left at
    their defaults (the library is one copy per process)."""
    lib.tp_last_error.restype = ctypes.c_char_p
    lib.tp_set_bn_flow.argtypes = [ctypes.c_int] * 4
    lib.tp_set_gemm_kmax.argtypes = [ctypes.c_int]
    lib.tp_set_gemm_twocta.argtypes = [ctypes.c_int]
    bad = [(lib.tp_set_bn_flow, (3, 0, 0, 0)), (lib.tp_set_bn_flow, (1, -1, 0, 0)),
           (lib.tp_set_bn_flow, (1, 0, 9, 0)), (lib.tp_set_bn_flow, (1, 0, 0, -5)),
           (lib.tp_set_gemm_kmax, (-1,)), (lib.tp_set_gemm_twocta, (3,))]
    for fn, args in bad:
        assert fn(*args) != 0, (fn, args)
        assert lib.tp_last_error(), (fn, args)
    assert lib.tp_set_bn_flow(0, 4, 2, 8192) == 0
    assert lib.tp_set_bn_flow(1, 0, 0, 0) == 0
    assert lib.tp_set_gemm_kmax(64) == 0
    assert lib.tp_set_gemm_twocta(1) == 0
