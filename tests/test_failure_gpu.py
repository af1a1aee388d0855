"""Failure detection on the GPU without a fault: a bounded in-kernel wait that runs out.

Every wait of the kernels on another unit's progress (an mbarrier phase of a TMA copy, an MMA
or an epilogue) is bounded in time.  Here the limit is lowered (``ff_set_wait_limit_ns``) so
that the GEMM's first wait for its operand tiles runs out: the kernel must record
FF_DEVICE_TIMEOUT in the device status word, drain its in-flight copies and MMAs, release
its tensor memory and return, and the next launch with the normal limit must compute the
right result.  Nothing here traps, faults or hangs: the drains keep the full 2 s limit."""
import numpy as np
import pytest
import torch

from firefly_b200 import _capi
from oracle import firefly_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_wait_timeout_sets_status_and_the_context_stays_usable():
    """K = 32768 keeps the epilogue warps waiting for the accumulator for tens of microseconds, far
    beyond a 1 microsecond limit (and beyond the resolution of the device timer), so their wait
    runs out on every CTA."""
    g = torch.Generator().manual_seed(5)
    M, N, K = 256, 128, 32768  # the 1-CTA kernel (128 x 64 tiles)
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    ad, bd = a.to(DEV), b.to(DEV)
    ref = _capi.gemm_i8(ad, bd, K, out_kind=_capi.FF_OUT_S32)
    assert _capi.device_status() == 0
    # the reference result itself, on a corner of the output (the full oracle product is slow)
    np.testing.assert_array_equal(ref[:8, :8].cpu().numpy().astype(np.int64), O.gemm_i8(a[:8].numpy(), b[:8].numpy()))
    lib = _capi.lib()
    assert lib.ff_set_wait_limit_ns(1000) == 0
    try:
        _capi.gemm_i8(ad, bd, K, out_kind=_capi.FF_OUT_S32)
        status = _capi.device_status()  # synchronises: the kernel returned
    finally:
        assert lib.ff_set_wait_limit_ns(0) == 0
    assert status & _capi.FF_DEVICE_TIMEOUT, status
    for _ in range(2):
        got = _capi.gemm_i8(ad, bd, K, out_kind=_capi.FF_OUT_S32)
        assert torch.equal(got, ref)
        assert _capi.device_status() == 0
