"""The C-ABI library loads without a GPU and exports every symbol include/*.h declares."""
import re
from pathlib import Path

import pytest

from firefly_b200 import _capi

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"^FF_API\s+[\w\s\*]+?\b(ff_\w+)\s*\(", h.read_text(), flags=re.M))
    return names


def test_header_declares_the_entry_points():
    names = _declared()
    assert {"ff_gemm_i8", "ff_quant_rows_i8", "ff_quant_dual_i8", "ff_dqt_adamw8", "ff_transpose_i8",
            "ff_version", "ff_last_error", "ff_device_status"} <= names


def test_library_exports_every_declared_symbol():
    lib = _capi.lib()
    for name in sorted(_declared()):
        assert hasattr(lib, name), name
    # the ctypes table covers exactly the declared functions
    assert set(_capi.SIGNATURES) == _declared()


def test_version_and_error_string():
    assert _capi.version().startswith("firefly_b200")
    assert "sm_100a" in _capi.version()
    assert isinstance(_capi.lib().ff_last_error(), bytes)


def test_argument_errors_need_no_gpu():
    """Bad arguments are rejected on the host before any CUDA call."""
    lib = _capi.lib()
    rc = lib.ff_gemm_i8(None, 16, None, 16, None, None, None, None, 8, 2, 8, 8, 0, None)
    assert rc == _capi.FF_ERR_INVALID_ARG
    assert b"K=0" in lib.ff_last_error()
    rc = lib.ff_dqt_adamw8(None, None, 8, 0, None, None, None, None, None, None, None, 512, 128,
                           1e-3, 0.9, 0.999, 1e-8, 0.0, 0.1, 0.001, 0.15, 0, 1, 0, None, None, None, None)
    assert rc == _capi.FF_ERR_UNSUPPORTED
    rc = lib.ff_quant_rows_i8(None, 7, 4, 4, 4, None, 1e-8, None, 4, None, None)
    assert rc == _capi.FF_ERR_INVALID_ARG
    # size-zero work is a no-op that succeeds
    assert lib.ff_quant_rows_i8(None, 0, 0, 4, 4, None, 1e-8, None, 4, None, None) == _capi.FF_OK
    assert lib.ff_gemm_i8(None, 16, None, 16, None, None, None, None, 8, 0, 0, 8, 16, None) == _capi.FF_OK


def test_no_cpu_fallback():
    """Product entry points refuse CPU tensors instead of computing on the host."""
    import torch
    with pytest.raises(RuntimeError):
        _capi.quant_rows(torch.zeros(2, 8))
    with pytest.raises(RuntimeError):
        _capi.gemm_i8(torch.zeros(2, 16, dtype=torch.int8), torch.zeros(2, 16, dtype=torch.int8), 16)


def test_noalloc_size_limit_checked_on_the_host_without_overflow():
    """The no-allocation dual quantiser refuses rows + cols above its built-in scratch before any
    CUDA call, also for sizes whose sum would overflow a signed 64-bit integer."""
    lib = _capi.lib()
    big = 2 ** 62
    for rows, cols in ((big, big), (2 ** 63 - 1, 1), (1, 2 ** 63 - 1), (262144, 1)):
        rc = lib.ff_quant_dual_i8_noalloc(None, _capi.FF_DTYPE_BF16, rows, cols, cols, None, 1e-8,
                                          None, 16, None, None, 16, None, None)
        assert rc == _capi.FF_ERR_UNSUPPORTED, (rows, cols)
        assert b"exceeds the built-in scratch" in lib.ff_last_error()


def test_gemm_workspace_size_and_argument_checks():
    """The split-K workspace size (no GPU needed), and the host-side refusal of a short one."""
    lib = _capi.lib()
    assert lib.ff_gemm_i8_ws_bytes(129, 8192, 8192) == 0
    assert lib.ff_gemm_i8_ws_bytes(0, 8192, 8192) == 0
    assert lib.ff_gemm_i8_ws_bytes(16, 8192, 8192) == 64 * 16 * 128 * 4 + 64 * 4
    assert lib.ff_gemm_i8_ws_bytes(128, 100, 64) == 1 * 128 * 128 * 4 + 4
    assert lib.ff_gemm_i8_ws_bytes(17, 8192, 64) == 64 * 32 * 128 * 4 + 64 * 4
