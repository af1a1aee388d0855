"""tcgen05 int8 GEMM against the oracle: int32 accumulators bit-exact, dequantised outputs
within 1e-3 relative (bf16: or within one bf16 step of the rounded oracle)."""
import numpy as np
import pytest
import torch

from firefly_b200 import _capi
from oracle import firefly_oracle as O
from tests._util import assert_close_rel, bf16_bits

pytestmark = pytest.mark.gpu
DEV = "cuda"
REL = 1e-3


def _operands(M, N, K, seed, ld_pad=0):
    g = torch.Generator().manual_seed(seed)
    lda = (K + 15) // 16 * 16 + ld_pad
    a = torch.zeros(M, lda, dtype=torch.int8)
    b = torch.zeros(N, lda, dtype=torch.int8)
    a[:, :K] = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    b[:, :K] = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    # garbage in the padding must not leak into the sums
    if lda > K:
        a[:, K:] = 77
        b[:, K:] = -55
    sa = torch.empty(M).uniform_(1e-3, 1e-2, generator=g)
    sb = torch.empty(N).uniform_(1e-3, 1e-2, generator=g)
    bias = torch.randn(N, generator=g)
    return a, b, sa, sb, bias


SHAPES = [
    (1, 1, 1),
    (128, 256, 128),
    (16, 512, 1024),
    (200, 300, 1000),
    (129, 257, 129),
    (256, 1024, 1024),
    (1024, 1024, 1024),
    (130, 8192, 256),
    (513, 200, 4096),
    (130, 18944, 512),    # 128 x 256 tiles, one CTA each
    (2600, 2600, 1000),   # 256 x 256 tiles on CTA pairs, ragged M, N and K
    (16, 8192, 8192),     # the skinny sizes of the GEMM sweep (HBM-bound: B streamed once)
    (128, 8192, 8192),
    (2560, 2048, 256),    # pair tiles with a short last wave, cut into 256 x 128 halves
    (2600, 1800, 384),    # the same with ragged M and N (one half tile entirely past N)
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_s32_bit_exact(M, N, K):
    a, b, *_ = _operands(M, N, K, seed=M + N + K, ld_pad=16 if K % 3 == 0 else 0)
    d = _capi.gemm_i8(a.to(DEV), b.to(DEV), K, out_kind=_capi.FF_OUT_S32)
    want = O.gemm_i8(a[:, :K].numpy(), b[:, :K].numpy())
    np.testing.assert_array_equal(d.cpu().numpy().astype(np.int64), want)
    assert _capi.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (200, 300, 1000), (256, 1024, 1024), (129, 257, 4096),
                                   (130, 18944, 512), (2600, 2600, 1000), (2600, 1800, 384)])
def test_gemm_f32_and_bf16_epilogue(M, N, K):
    a, b, sa, sb, bias = _operands(M, N, K, seed=3 * M + K)
    acc = O.gemm_i8(a[:, :K].numpy(), b[:, :K].numpy())
    want = O.dequant(acc, sa.numpy(), sb.numpy(), bias.numpy())
    ad, bd = a.to(DEV), b.to(DEV)
    d32 = _capi.gemm_i8(ad, bd, K, sa.to(DEV), sb.to(DEV), bias.to(DEV), out_kind=_capi.FF_OUT_F32)
    # same fp32 operation order as the oracle: identical results expected
    np.testing.assert_array_equal(d32.cpu().numpy(), want)
    d16 = _capi.gemm_i8(ad, bd, K, sa.to(DEV), sb.to(DEV), bias.to(DEV), out_kind=_capi.FF_OUT_BF16)
    want16 = O.f32_to_bf16_bits(want)
    np.testing.assert_array_equal(bf16_bits(d16), want16)
    # scale_a only (the dX epilogue)
    d = _capi.gemm_i8(ad, bd, K, sa.to(DEV), None, None, out_kind=_capi.FF_OUT_F32)
    np.testing.assert_array_equal(d.cpu().numpy(), O.dequant(acc, sa.numpy()))
    assert_close_rel(d.cpu().numpy(), O.dequant(acc, sa.numpy()), REL, "scale_a only")


@pytest.mark.parametrize("M,N,K", [(300, 520, 700), (2600, 2600, 1000)])
def test_gemm_bf16_accumulate(M, N, K):
    a, b, sa, sb, _ = _operands(M, N, K, seed=5)
    g = torch.Generator().manual_seed(6)
    old = torch.randn(M, N, generator=g).to(torch.bfloat16)
    d = old.clone().to(DEV)
    _capi.gemm_i8(a.to(DEV), b.to(DEV), K, sa.to(DEV), sb.to(DEV), out_kind=_capi.FF_OUT_BF16_ACCUM, out=d)
    acc = O.gemm_i8(a[:, :K].numpy(), b[:, :K].numpy())
    term = O.round_bf16(O.dequant(acc, sa.numpy(), sb.numpy()))
    want = O.f32_to_bf16_bits(old.float().numpy() + term)
    np.testing.assert_array_equal(bf16_bits(d), want)


def test_gemm_strided_output_and_misaligned_n():
    M, N, K = 70, 45, 96
    a, b, sa, sb, bias = _operands(M, N, K, seed=8)
    big = torch.zeros(M, 64, dtype=torch.float32, device=DEV)
    out = big[:, 3:3 + N]
    _capi.gemm_i8(a.to(DEV), b.to(DEV), K, sa.to(DEV), sb.to(DEV), bias.to(DEV), out_kind=_capi.FF_OUT_F32, out=out)
    acc = O.gemm_i8(a[:, :K].numpy(), b[:, :K].numpy())
    np.testing.assert_array_equal(out.cpu().numpy(), O.dequant(acc, sa.numpy(), sb.numpy(), bias.numpy()))
    assert (big[:, :3] == 0).all() and (big[:, 3 + N:] == 0).all()


def test_gemm_rejects_bad_layout():
    a = torch.zeros(4, 24, dtype=torch.int8, device=DEV)
    b = torch.zeros(4, 32, dtype=torch.int8, device=DEV)
    with pytest.raises(ValueError):
        _capi.gemm_i8(a, b, 24, out_kind=_capi.FF_OUT_S32)  # lda = 24 is not a multiple of 16
    with pytest.raises(ValueError):
        _capi.gemm_i8(b, b, 0, out_kind=_capi.FF_OUT_S32)


def test_gemm_large_square_checksum():
    """8192^3 (the headline size): exact int32 checked through size-independent properties.

    acc = A·Bᵀ; for all-ones x, (A·Bᵀ)·x = A·(Bᵀ·x) checked in int64 on the host, and a
    random sample of entries is recomputed exactly."""
    M = N = K = 8192
    g = torch.Generator(device=DEV).manual_seed(0)
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8, device=DEV)
    b = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8, device=DEV)
    d = _capi.gemm_i8(a, b, K, out_kind=_capi.FF_OUT_S32)
    row_sums = d.to(torch.int64).sum(dim=1)
    bt_ones = b.to(torch.int64).sum(dim=0)  # Bᵀ·1, [K]
    want = (a.to(torch.int64) * bt_ones[None, :]).sum(dim=1)
    assert torch.equal(row_sums, want)
    idx = torch.randint(0, M, (64,), generator=torch.Generator().manual_seed(1))
    jdx = torch.randint(0, N, (64,), generator=torch.Generator().manual_seed(2))
    ai = a[idx.to(DEV)].to(torch.int64).cpu()
    bj = b[jdx.to(DEV)].to(torch.int64).cpu()
    sub = d[idx.to(DEV)][:, jdx.to(DEV)].to(torch.int64).cpu()
    assert torch.equal(sub, ai @ bj.T)
    assert _capi.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (200, 300, 1000), (8192, 4096, 1100), (2600, 2600, 1000),
                                   (130, 18944, 512), (64, 96, 70)])
def test_gemm_kn_layout_bit_exact(M, N, K):
    """B given K x N row-major (the dX GEMM reads W [O, K_in] this way): MN-major staging."""
    g = torch.Generator().manual_seed(M + 3 * N + K)
    ldb = (N + 15) // 16 * 16
    a = torch.zeros(M, (K + 15) // 16 * 16, dtype=torch.int8)
    a[:, :K] = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    b = torch.zeros(K, ldb, dtype=torch.int8)
    b[:, :N] = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int8)
    b[:, N:] = 99  # padding columns must not leak
    sa = torch.empty(M).uniform_(1e-3, 1e-2, generator=g)
    d = _capi.gemm_i8(a.to(DEV), b.to(DEV), K, out_kind=_capi.FF_OUT_S32, b_kn_cols=N)
    acc = O.gemm_i8(a[:, :K].numpy(), np.ascontiguousarray(b[:, :N].numpy().T))
    np.testing.assert_array_equal(d.cpu().numpy().astype(np.int64), acc)
    d16 = _capi.gemm_i8(a.to(DEV), b.to(DEV), K, sa.to(DEV), out_kind=_capi.FF_OUT_BF16, b_kn_cols=N)
    np.testing.assert_array_equal(bf16_bits(d16), O.f32_to_bf16_bits(O.dequant(acc, sa.numpy())))
    assert _capi.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(16, 8192, 8192), (128, 8192, 8192), (33, 1000, 3000), (100, 130, 640),
                                   (64, 256, 128)])
def test_skinny_split_k_equals_oracle_and_leaves_workspace_zero(M, N, K):
    """Skinny A (M <= 128) runs stream-K with a split-K workspace: int32 results bit-exact, the
    scaled epilogues identical to the unsplit kernel (ff_gemm_i8 without a workspace), and the
    workspace all zeros again after every call, so a second call gives the same results."""
    import ctypes

    a, b, sa, sb, bias = _operands(M, N, K, seed=7 * M + N)
    ad, bd = a.to(DEV), b.to(DEV)
    lib = _capi.lib()
    need = lib.ff_gemm_i8_ws_bytes(M, N, K)
    assert need == -(-N // 128) * (16 if M <= 16 else 32 if M <= 32 else 64 if M <= 64 else 128) * 128 * 4 \
        + -(-N // 128) * 4
    ws = torch.zeros(need + 16, dtype=torch.uint8, device=DEV)
    want = O.gemm_i8(a[:, :K].numpy(), b[:, :K].numpy())
    lda = a.shape[1]
    for kind in (_capi.FF_OUT_S32, _capi.FF_OUT_F32, _capi.FF_OUT_BF16):
        odt = {_capi.FF_OUT_S32: torch.int32, _capi.FF_OUT_F32: torch.float32, _capi.FF_OUT_BF16: torch.bfloat16}[kind]
        ref = torch.empty(M, N, dtype=odt, device=DEV)
        sa_d, sb_d, bias_d = sa.to(DEV), sb.to(DEV), bias.to(DEV)
        args = (ctypes.c_void_p(ad.data_ptr()), lda, ctypes.c_void_p(bd.data_ptr()), lda,
                ctypes.c_void_p(sa_d.data_ptr()), ctypes.c_void_p(sb_d.data_ptr()), ctypes.c_void_p(bias_d.data_ptr()))
        assert lib.ff_gemm_i8(*args, ctypes.c_void_p(ref.data_ptr()), N, kind, M, N, K, None) == 0
        for _ in range(2):
            got = torch.full((M, N), 7, dtype=odt, device=DEV)
            rc = lib.ff_gemm_i8_ws(*args, ctypes.c_void_p(got.data_ptr()), N, kind, M, N, K,
                                   ctypes.c_void_p(ws.data_ptr()), need, None)
            assert rc == 0, lib.ff_last_error()
            torch.cuda.synchronize()
            assert torch.equal(got, ref), kind
            assert int(ws.count_nonzero()) == 0
        if kind == _capi.FF_OUT_S32:
            np.testing.assert_array_equal(got.cpu().numpy().astype(np.int64), want)
    assert _capi.device_status() == 0
