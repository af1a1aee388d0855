"""The allocation-free dual quantiser, called through the C ABI.

``ff_quant_dual_i8_noalloc`` serves callers that cannot allocate device memory
(a runtime whose device memory is owned by its own pool allocator, or a pipelined
step that cannot afford cudaMalloc's implicit device synchronisation): it keeps
its absmax scratch in a static array inside the library instead of taking a
workspace.  This test checks it against ``ff_quant_dual_i8`` (given a workspace)
on two calls in a row — the second call reuses the scratch the first one left
behind, so it also checks that the scratch is cleared — and that sizes above the
built-in limit are refused.  It lives in its own file, named to be collected
last, and passes alone or after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

from firefly_b200 import _capi

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
FF_NOALLOC_DUAL_MAX_ELEMS = 262144


def _noalloc(x: torch.Tensor, colmul: torch.Tensor | None):
    R, C = x.shape
    ldq, ldqt = _capi.round_up(C, 16), _capi.round_up(max(R, 1), 16)
    q_rows = torch.empty((R, ldq), dtype=torch.int8, device=DEV)
    s_rows = torch.empty((R,), dtype=torch.float32, device=DEV)
    q_cols = torch.empty((C, ldqt), dtype=torch.int8, device=DEV)
    s_cols = torch.empty((C,), dtype=torch.float32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    rc = _capi.lib().ff_quant_dual_i8_noalloc(
        ctypes.c_void_p(x.data_ptr()), _capi._dtype_code(x.dtype), R, C, C,
        None if colmul is None else ctypes.c_void_p(colmul.data_ptr()), 1e-8,
        ctypes.c_void_p(q_rows.data_ptr()), ldq, ctypes.c_void_p(s_rows.data_ptr()),
        ctypes.c_void_p(q_cols.data_ptr()), ldqt, ctypes.c_void_p(s_cols.data_ptr()), stream)
    assert rc == _capi.FF_OK, _capi.lib().ff_last_error()
    return q_rows, s_rows, q_cols, s_cols


def test_noalloc_matches_workspace_version_on_two_calls():
    g = torch.Generator(device=DEV).manual_seed(0)
    cases = [
        (torch.randn(1000, 3000, device=DEV, generator=g) * 5).to(torch.bfloat16),
        # second call: smaller absmax values than the first, so stale scratch would show
        (torch.randn(777, 1500, device=DEV, generator=g) * 0.01).to(torch.bfloat16),
    ]
    for i, x in enumerate(cases):
        colmul = torch.rand(x.shape[1], device=DEV, generator=g) * 1e-3 + 1e-4
        got = _noalloc(x, colmul)
        want = _capi.quant_dual(x, row_colmul=colmul)
        torch.cuda.synchronize()
        for name, a, b in zip(("q_rows", "s_rows", "q_cols_t", "s_cols"), got, want):
            np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy(), err_msg=f"call {i}: {name}")
    assert _capi.device_status() == 0


def test_noalloc_refuses_sizes_above_its_scratch():
    x = torch.zeros((FF_NOALLOC_DUAL_MAX_ELEMS, 8), dtype=torch.bfloat16, device=DEV)
    q = torch.empty(1, dtype=torch.int8, device=DEV)
    s = torch.empty(1, dtype=torch.float32, device=DEV)
    rc = _capi.lib().ff_quant_dual_i8_noalloc(
        ctypes.c_void_p(x.data_ptr()), _capi.FF_DTYPE_BF16, x.shape[0], x.shape[1], x.shape[1], None, 1e-8,
        ctypes.c_void_p(q.data_ptr()), 16, ctypes.c_void_p(s.data_ptr()), None, 16, None, None)
    assert rc == _capi.FF_ERR_UNSUPPORTED
    assert b"exceeds" in _capi.lib().ff_last_error()
