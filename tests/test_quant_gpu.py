"""Quantiser and transpose kernels against the oracle (bit-exact integer codes)."""
import numpy as np
import pytest
import torch

from firefly_b200 import _capi, quantize_fp_to_int8
from oracle import firefly_oracle as O
from tests._util import load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rand(shape, dtype, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


def test_quantize_fp_to_int8_golden():
    """The kernel reproduces the reference's own quantize_fp_to_int8 outputs bit for bit."""
    z = load_golden("quant_rows.npz")
    cases = sorted({k[:-2] for k in z.files if k.endswith("_q")})
    for c in cases:
        x = torch.from_numpy(z[c + "_x"])
        if bool(z[c + "_isbf16"]):
            x = x.to(torch.bfloat16)
        eps = 1e-5 if c == "eps" else 1e-8
        q, s = quantize_fp_to_int8(x.to(DEV), eps=eps)
        np.testing.assert_array_equal(q.cpu().numpy(), z[c + "_q"], err_msg=c)
        np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), z[c + "_s"].view(np.uint32), err_msg=c)
        # CPU input: quantised on the GPU, returned on the CPU
        q2, s2 = quantize_fp_to_int8(x, eps=eps)
        assert q2.device.type == "cpu"
        np.testing.assert_array_equal(q2.numpy(), z[c + "_q"], err_msg=c)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(1, 1), (7, 13), (33, 300), (256, 1024), (5, 4104), (130, 2050)])
def test_quant_rows_matches_oracle(dtype, shape):
    x = _rand(shape, dtype, seed=shape[0] * 7 + shape[1])
    x[0, :] = 0  # an all-zero row (eps clamp)
    q, s = _capi.quant_rows(x.to(DEV))
    qo, so = O.quantize_rows(x.float().numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))


def test_quant_rows_padding_colmul_and_strides():
    x = _rand((40, 100), torch.bfloat16, seed=3)
    cm = torch.rand(100, generator=torch.Generator().manual_seed(4)) * 0.01
    q, s = _capi.quant_rows(x.to(DEV), colmul=cm.to(DEV), ldq=112)
    qo, so = O.quantize_rows(x.float().numpy(), colmul=cm.numpy())
    qc = q.cpu().numpy()
    np.testing.assert_array_equal(qc[:, :100], qo)
    assert (qc[:, 100:] == 0).all()
    np.testing.assert_array_equal(s.cpu().numpy(), so)
    # a strided (non-contiguous rows) input view
    big = _rand((40, 160), torch.float32, seed=5).to(DEV)
    view = big[:, 8:108]
    q, s = _capi.quant_rows(view)
    qo, so = O.quantize_rows(view.cpu().numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), qo)


def test_quant_rows_ties_and_extremes():
    x = torch.zeros(3, 64)
    x[:, 0] = 127.0
    x[0, 1:33] = torch.arange(32) + 0.5  # exact .5 ties: round half to even
    x[1, 1:] = torch.linspace(-1e30, 1e30, 63)
    x[2, 1:] = torch.linspace(-1e-30, 1e-30, 63)
    q, s = _capi.quant_rows(x.to(DEV))
    qo, so = O.quantize_rows(x.numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)


def test_quant_rows_empty_and_bad_args():
    q, s = _capi.quant_rows(torch.zeros(0, 9, device=DEV))
    assert q.shape == (0, 9) and s.shape == (0,)
    with pytest.raises(ValueError):
        _capi.quant_rows(torch.zeros(4, 0, device=DEV))
    with pytest.raises(ValueError):
        quantize_fp_to_int8(torch.zeros(3, device=DEV))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 1), (17, 33), (256, 1024), (300, 130), (129, 1030), (1000, 16)])
def test_quant_dual_matches_oracle(dtype, shape):
    x = _rand(shape, dtype, seed=11 + shape[0])
    R, C = shape
    x[min(1, R - 1), :] = 0
    cm = torch.rand(C, generator=torch.Generator().manual_seed(12)) * 1e-3 + 1e-4
    q_r, s_r, q_t, s_t = _capi.quant_dual(x.to(DEV), row_colmul=cm.to(DEV))
    xf = x.float().numpy()
    qo, so = O.quantize_rows(xf, colmul=cm.numpy())
    qto, sto = O.quantize_cols_t(xf)
    qr = q_r.cpu().numpy()
    np.testing.assert_array_equal(qr[:, :C], qo)
    assert (qr[:, C:] == 0).all()
    np.testing.assert_array_equal(s_r.cpu().numpy(), so)
    qt = q_t.cpu().numpy()
    np.testing.assert_array_equal(qt[:, :R], qto)
    assert (qt[:, R:] == 0).all()
    np.testing.assert_array_equal(s_t.cpu().numpy(), sto)


def test_quant_dual_one_side_only():
    x = _rand((70, 90), torch.bfloat16, seed=21).to(DEV)
    q_r, s_r, q_t, s_t = _capi.quant_dual(x, rows=False, cols=True)
    assert q_r is None and s_r is None
    qto, sto = O.quantize_cols_t(x.float().cpu().numpy())
    np.testing.assert_array_equal(q_t.cpu().numpy()[:, :70], qto)
    q_r, s_r, q_t, s_t = _capi.quant_dual(x, rows=True, cols=False)
    assert q_t is None
    qo, so = O.quantize_rows(x.float().cpu().numpy())
    np.testing.assert_array_equal(q_r.cpu().numpy()[:, :90], qo)


@pytest.mark.parametrize("shape", [(1, 1), (64, 64), (100, 37), (1024, 4096), (4099, 70)])
def test_transpose_i8(shape):
    g = torch.Generator().manual_seed(shape[0])
    w = torch.randint(-127, 128, shape, generator=g, dtype=torch.int8)
    t = _capi.transpose_i8(w.to(DEV))
    R, C = shape
    tc = t.cpu().numpy()
    assert tc.shape == (C, (R + 15) // 16 * 16)
    np.testing.assert_array_equal(tc[:, :R], w.numpy().T)
    assert (tc[:, R:] == 0).all()


def test_colsum_bf16():
    x = _rand((1000, 77), torch.bfloat16, seed=31).to(DEV)
    got = _capi.colsum_bf16(x)
    want = O.f32_to_bf16_bits(x.float().cpu().numpy().astype(np.float64).sum(0).astype(np.float32))
    gb = got.cpu().view(torch.int16).numpy().view(np.uint16)
    from tests._util import bf16_ulp_diff
    assert bf16_ulp_diff(gb, want).max() <= 1
    # deterministic
    np.testing.assert_array_equal(gb, _capi.colsum_bf16(x).cpu().view(torch.int16).numpy().view(np.uint16))


@pytest.mark.parametrize("shape,colmul,rows", [((1000, 77), False, True), ((1, 5), False, True),
                                               ((129, 1030), True, True), ((300, 2050), True, False),
                                               ((4096, 512), False, True), ((0, 24), False, True)])
def test_quant_dual_with_column_sums(shape, colmul, rows):
    """quant_dual(colsum=True): the same codes and scales as quant_dual, plus the bias
    gradient Σ_r x[r, :] within 1 bf16 ulp of the exact sum, deterministic."""
    from tests._util import bf16_ulp_diff
    R, C = shape
    x = _rand(shape, torch.bfloat16, seed=R * 3 + C).to(DEV)
    cm = (torch.rand(C, generator=torch.Generator().manual_seed(C)) + 0.5).to(DEV) if colmul else None
    got = _capi.quant_dual(x, row_colmul=cm, rows=rows, colsum=True)
    if R:
        want = _capi.quant_dual(x, row_colmul=cm, rows=rows)
        for a, b in zip(got[:4], want):
            assert (a is None) == (b is None)
            if a is not None:
                np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
    exact = O.f32_to_bf16_bits(x.float().cpu().numpy().astype(np.float64).sum(0).astype(np.float32))
    db = got[4].cpu().view(torch.int16).numpy().view(np.uint16)
    assert db.shape == (C,)
    assert bf16_ulp_diff(db, exact).max() <= 1
    again = _capi.quant_dual(x, row_colmul=cm, rows=rows, colsum=True)[4]
    np.testing.assert_array_equal(db, again.cpu().view(torch.int16).numpy().view(np.uint16))


def test_quant_dual_column_sums_need_bf16():
    with pytest.raises(ValueError):
        _capi.quant_dual(torch.zeros((4, 8), dtype=torch.float32, device=DEV), colsum=True)


def test_update_int8_weight():
    g = torch.Generator().manual_seed(9)
    w = torch.randint(-127, 128, (50, 60), generator=g, dtype=torch.int8)
    dq = torch.randint(-300, 300, (50, 60), generator=g, dtype=torch.int32)
    wd = w.to(DEV)
    from firefly_b200.fireflykernels import update_int8_weight_
    update_int8_weight_(wd, dq.to(DEV))
    want = (w.to(torch.int16) + dq.to(torch.int16)).clamp(-127, 127).to(torch.int8)
    np.testing.assert_array_equal(wd.cpu().numpy(), want.numpy())
