"""SwiGLU producer fusion: the fused quantisers and the fused MLP op.

* ``ff_swiglu_quant_i8`` must give exactly torch's bf16 ``h = F.silu(g) * u`` and
  ``quant_dual(h)``;
* ``ff_swiglu_bwd_quant_i8`` must give exactly ``[dg | du]`` from torch's autograd of
  ``F.silu(g) * u`` and ``quant_dual([dg | du], colmul)``;
* ``SwiGLUMLP`` (fused op) must match the composition of BitLinear layers and torch's
  elementwise ops bit for bit, and the oracle's ``swiglu_mlp_step``.
"""
import numpy as np
import pytest
import torch
from torch.nn import functional as F

from firefly_b200 import _capi
from firefly_b200.swiglu import SwiGLUMLP
from oracle import firefly_oracle as O
from tests._util import assert_close_rel, bf16_bits, bf16_ulp_diff, from_bf16_bits

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
NAMES = ("q_rows", "s_rows", "q_cols_t", "s_cols")


def _gu(T, Fh, seed, scale=3.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(T, 2 * Fh, device=DEV, generator=g) * scale).to(torch.bfloat16)


def test_swiglu_arithmetic_exact_for_every_bf16_input():
    """The kernels' branch-free 1/(1+exp(-x)) and x/(1+exp(-x)) equal torch's IEEE divides
    for all 65536 bf16 x (the inputs outside the fast path's range take IEEE ops)."""
    mism, ieee, first = _capi.swiglu_selftest()
    x = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        # outside the fast path: x not finite, or 1 + exp(-x) >= 2^126 (x <= -87.34)
        out_of_range = int((~np.isfinite(x) | (np.exp(-x.astype(np.float64)) >= 2.0 ** 126)).sum())
    assert mism == 0, f"{mism} mismatches, first bf16 pattern {first:#06x}"
    assert ieee == out_of_range


def test_swiglu_exhaustive_through_the_kernels():
    """Every bf16 gate value through both fused kernels against torch (u, dh varied)."""
    allg = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).to(DEV)
    gen = torch.Generator(device=DEV).manual_seed(3)
    T, Fh = 256, 256
    g = allg.view(T, Fh)
    fin = torch.isfinite(g)
    g = torch.where(fin, g, torch.zeros_like(g))  # inf/nan gates would make whole rows non-finite
    u = torch.randn(T, Fh, device=DEV, generator=gen).to(torch.bfloat16)
    gu = torch.cat([g, u], dim=1).requires_grad_(True)
    dh = torch.randn(T, Fh, device=DEV, generator=gen).to(torch.bfloat16)
    gg, uu = gu.chunk(2, dim=1)
    h = F.silu(gg) * uu
    h.backward(dh)
    got = _capi.swiglu_quant(gu.detach())
    np.testing.assert_array_equal(bf16_bits(got[4]), bf16_bits(h), err_msg="h")
    _assert_same(got, _capi.quant_dual(h), "forward codes")
    gotb = _capi.swiglu_bwd_quant(dh, gu.detach())
    np.testing.assert_array_equal(bf16_bits(gotb[4]), bf16_bits(gu.grad), err_msg="[dg | du]")
    _assert_same(gotb, _capi.quant_dual(gu.grad), "backward codes")


def _assert_same(got, want, what):
    for name, a, b in zip(NAMES, got, want):
        assert a.shape == b.shape, f"{what} {name}: {tuple(a.shape)} vs {tuple(b.shape)}"
        np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy(), err_msg=f"{what}: {name}")


@pytest.mark.parametrize("T,Fh", [(256, 1376), (37, 40), (1, 16), (130, 24), (33, 13), (129, 1000)])
def test_swiglu_quant_matches_quant_dual_of_torch_h(T, Fh):
    gu = _gu(T, Fh, seed=T + Fh)
    g, u = gu.chunk(2, dim=1)
    h = F.silu(g) * u
    want = _capi.quant_dual(h)
    got = _capi.swiglu_quant(gu)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bf16_bits(got[4]), bf16_bits(h), err_msg="h")
    _assert_same(got, want, f"T={T} f={Fh}")
    # row part only / column part only
    q, s, qt, st, _ = _capi.swiglu_quant(gu, cols=False)
    assert qt is None and st is None
    np.testing.assert_array_equal(q.cpu().numpy(), want[0].cpu().numpy())
    q, s, qt, st, _ = _capi.swiglu_quant(gu, rows=False)
    assert q is None and s is None
    np.testing.assert_array_equal(qt.cpu().numpy(), want[2].cpu().numpy())
    assert _capi.device_status() == 0


@pytest.mark.parametrize("T,Fh,colmul", [(256, 1376, True), (37, 48, True), (1, 16, False), (300, 32, False),
                                         (45, 1000, True), (3, 8, True)])
def test_swiglu_bwd_quant_matches_torch_autograd(T, Fh, colmul):
    gu = _gu(T, Fh, seed=2 * T + Fh).requires_grad_(True)
    gen = torch.Generator(device=DEV).manual_seed(T)
    dh = torch.randn(T, Fh, device=DEV, generator=gen).to(torch.bfloat16)
    g, u = gu.chunk(2, dim=1)
    (F.silu(g) * u).backward(dh)
    cm = torch.rand(2 * Fh, device=DEV, generator=gen) * 1e-2 + 1e-4 if colmul else None
    want = _capi.quant_dual(gu.grad, row_colmul=cm)
    got = _capi.swiglu_bwd_quant(dh, gu.detach(), colmul=cm)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bf16_bits(got[4]), bf16_bits(gu.grad), err_msg="[dg | du]")
    _assert_same(got, want, f"T={T} f={Fh}")
    q, s, qt, st, _ = _capi.swiglu_bwd_quant(dh, gu.detach(), colmul=cm, rows=False)
    assert q is None
    np.testing.assert_array_equal(qt.cpu().numpy(), want[2].cpu().numpy())
    assert _capi.device_status() == 0


@pytest.mark.parametrize("T,F,K", [(256, 256, 512), (37, 128, 64), (300, 384, 1000), (1024, 1408, 4096),
                                   (1, 128, 16)])
def test_swiglu_gemm_epilogue_matches_gemm_then_quantiser(T, F, K):
    """The gate/up GEMM with h in its epilogue equals ff_gemm_i8 (bf16 out) followed by
    ff_swiglu_quant_i8, bit for bit: gu, h and all codes and scales."""
    gen = torch.Generator(device=DEV).manual_seed(T + F + K)
    ldk = _capi.round_up(K, 16)
    a = torch.zeros(T, ldk, dtype=torch.int8, device=DEV)
    a[:, :K] = torch.randint(-127, 128, (T, K), dtype=torch.int8, device=DEV, generator=gen)
    w = torch.zeros(2 * F, ldk, dtype=torch.int8, device=DEV)
    w[:, :K] = torch.randint(-127, 128, (2 * F, K), dtype=torch.int8, device=DEV, generator=gen)
    sa = torch.rand(T, device=DEV, generator=gen) * 2e-2 + 1e-3
    sb = torch.rand(2 * F, device=DEV, generator=gen) * 2e-3 + 1e-4
    gu_ref = _capi.gemm_i8(a, w, K, scale_a=sa, scale_b=sb, out_kind=_capi.FF_OUT_BF16)
    want = _capi.swiglu_quant(gu_ref)
    gu, *got = _capi.swiglu_gemm(a, w, K, sa, sb)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bf16_bits(gu), bf16_bits(gu_ref), err_msg="gu")
    np.testing.assert_array_equal(bf16_bits(got[4]), bf16_bits(want[4]), err_msg="h")
    _assert_same(got[:4], want[:4], f"T={T} F={F} K={K}")
    # row codes only (the forward without gradient)
    _, q, s_, qt, st, _ = _capi.swiglu_gemm(a, w, K, sa, sb, cols=False)
    assert qt is None
    np.testing.assert_array_equal(q.cpu().numpy(), want[0].cpu().numpy())
    assert _capi.device_status() == 0


@pytest.mark.parametrize("T,F,O,colmul", [(256, 256, 512, True), (37, 128, 64, True), (300, 384, 1000, False),
                                         (1024, 1408, 4096, True), (1, 128, 16, True)])
def test_swiglu_bwd_gemm_epilogue_matches_gemm_then_quantiser(T, F, O, colmul):
    """dH GEMM with the SwiGLU backward in its epilogue equals ff_gemm_i8_kn (bf16 dh)
    followed by ff_swiglu_bwd_quant_i8, bit for bit."""
    gen = torch.Generator(device=DEV).manual_seed(T + F + O)
    ldo = _capi.round_up(O, 16)
    a = torch.zeros(T, ldo, dtype=torch.int8, device=DEV)
    a[:, :O] = torch.randint(-127, 128, (T, O), dtype=torch.int8, device=DEV, generator=gen)
    w = torch.randint(-127, 128, (O, F), dtype=torch.int8, device=DEV, generator=gen)
    sa = torch.rand(T, device=DEV, generator=gen) * 2e-3 + 1e-4
    gu = _gu(T, F, seed=T + 3)
    cm = torch.rand(2 * F, device=DEV, generator=gen) * 1e-2 + 1e-4 if colmul else None
    dh = _capi.gemm_i8(a, w, O, scale_a=sa, out_kind=_capi.FF_OUT_BF16, b_kn_cols=F)
    want = _capi.swiglu_bwd_quant(dh, gu, colmul=cm)
    got = _capi.swiglu_bwd_gemm(a, w, O, sa, gu, colmul=cm)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bf16_bits(got[4]), bf16_bits(want[4]), err_msg="[dg | du]")
    _assert_same(got[:4], want[:4], f"T={T} F={F} O={O}")
    q, s_, qt, st, _ = _capi.swiglu_bwd_gemm(a, w, O, sa, gu, colmul=cm, rows=False)
    assert q is None
    np.testing.assert_array_equal(qt.cpu().numpy(), want[2].cpu().numpy())
    assert _capi.device_status() == 0


def test_swiglu_gemm_with_bias_and_extreme_gates():
    """Bias in the epilogue, and gate values beyond the fast path's range (IEEE fallback)."""
    T, F, K = 128, 128, 64
    gen = torch.Generator(device=DEV).manual_seed(1)
    a = torch.randint(-127, 128, (T, K), dtype=torch.int8, device=DEV, generator=gen)
    w = torch.randint(-127, 128, (2 * F, K), dtype=torch.int8, device=DEV, generator=gen)
    sa = torch.rand(T, device=DEV, generator=gen) * 1e-1
    sb = torch.rand(2 * F, device=DEV, generator=gen) * 1e-1
    sb[:F:7] *= 100.0  # some gate columns reach |g| > 87
    bias = torch.randn(2 * F, device=DEV, generator=gen)
    gu_ref = _capi.gemm_i8(a, w, K, scale_a=sa, scale_b=sb, bias=bias, out_kind=_capi.FF_OUT_BF16)
    assert (gu_ref[:, :F].float() < -87.4).any()
    want = _capi.swiglu_quant(gu_ref)
    gu, *got = _capi.swiglu_gemm(a, w, K, sa, sb, bias=bias)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bf16_bits(gu), bf16_bits(gu_ref), err_msg="gu")
    np.testing.assert_array_equal(bf16_bits(got[4]), bf16_bits(want[4]), err_msg="h")
    _assert_same(got[:4], want[:4], "bias")


def test_oracle_swiglu_formulas_match_torch():
    """The oracle's restatement of torch's bf16 silu/mul and their autograd formulas."""
    T, Fh = 512, 512
    gu = _gu(T, Fh, seed=5, scale=4.0).requires_grad_(True)
    dh = torch.randn(T, Fh, device=DEV, generator=torch.Generator(device=DEV).manual_seed(6)).to(torch.bfloat16)
    g, u = gu.chunk(2, dim=1)
    h = F.silu(g) * u
    h.backward(dh)
    gf = O.bf16_bits_to_f32(bf16_bits(g))
    uf = O.bf16_bits_to_f32(bf16_bits(u))
    dhf = O.bf16_bits_to_f32(bf16_bits(dh))
    h_o = O.f32_to_bf16_bits(O.swiglu_forward(gf, uf))
    dg_o, du_o = (O.f32_to_bf16_bits(a) for a in O.swiglu_backward(dhf, gf, uf))
    grad = gu.grad
    for what, got, want in (("h", bf16_bits(h), h_o), ("dg", bf16_bits(grad[:, :Fh]), dg_o),
                            ("du", bf16_bits(grad[:, Fh:]), du_o)):
        d = bf16_ulp_diff(got, want)
        # exp is correctly rounded here and within 2 ulp in CUDA: rare one-step bf16 flips
        assert d.max() <= 1, what
        assert (d > 0).mean() <= 1e-3, f"{what}: {(d > 0).mean():.2e} of elements differ"


def test_swiglu_bwd_rejects_unaligned_ffn():
    gu = _gu(8, 20, seed=1)
    dh = torch.zeros(8, 20, dtype=torch.bfloat16, device=DEV)
    with pytest.raises((ValueError, RuntimeError), match="multiple of 8"):
        _capi.swiglu_bwd_quant(dh, gu)


def _pair(d, f, seed):
    torch.manual_seed(seed)
    fused = SwiGLUMLP(d, f).to(DEV)
    fused.init_normal_(0.02, generator=torch.Generator(device=DEV).manual_seed(seed))
    plain = SwiGLUMLP(d, f, fused=False).to(DEV)
    with torch.no_grad():
        for a, b in ((fused.gate_up, plain.gate_up), (fused.down, plain.down)):
            b.int_weight.copy_(a.int_weight)
            b.weight_scale.copy_(a.weight_scale)
    return fused, plain


@pytest.mark.parametrize("T,d,f,xdt", [(200, 256, 512, torch.bfloat16), (37, 96, 80, torch.float32),
                                       (1, 32, 16, torch.bfloat16), (50, 40, 24, torch.bfloat16),
                                       (20, 48, 20, torch.bfloat16), (300, 64, 128, torch.float32)])
def test_fused_mlp_matches_unfused_composition(T, d, f, xdt):
    fused, plain = _pair(d, f, seed=T + d)
    gen = torch.Generator(device=DEV).manual_seed(9)
    x = torch.randn(T, d, device=DEV, generator=gen).to(xdt)
    dy = torch.randn(T, d, device=DEV, generator=gen).to(torch.bfloat16)
    outs = []
    for m in (fused, plain):
        xi = x.clone().requires_grad_(True)
        y = m(xi)
        y.backward(dy)
        outs.append((y, xi.grad, m.gate_up.consume_weight_grad(), m.down.consume_weight_grad()))
    for what, a, b in zip(("y", "dx", "dW gate_up", "dW down"), *outs):
        assert a.dtype == b.dtype and a.shape == b.shape, what
        np.testing.assert_array_equal(bf16_bits(a), bf16_bits(b), err_msg=what)
    assert _capi.device_status() == 0


def test_fused_mlp_matches_oracle():
    T, d, f = 96, 128, 160
    fused, _ = _pair(d, f, seed=11)
    gen = torch.Generator().manual_seed(12)
    x = torch.randn(T, d, generator=gen).to(torch.bfloat16)
    dy = torch.randn(T, d, generator=gen).to(torch.bfloat16)
    xd = x.to(DEV).requires_grad_(True)
    y = fused(xd)
    y.backward(dy.to(DEV))
    q_gu, s_gu = fused.gate_up.int_weight.cpu().numpy(), fused.gate_up.weight_scale.cpu().numpy()
    q_d, s_d = fused.down.int_weight.cpu().numpy(), fused.down.weight_scale.cpu().numpy()
    want = O.swiglu_mlp_step(x.float().numpy(), bf16_bits(dy), q_gu, s_gu, q_d, s_d)
    for what, got, key in (("y", y, "y"), ("dx", xd.grad, "dx"),
                           ("dW gate_up", fused.gate_up.consume_weight_grad(), "gw_gu"),
                           ("dW down", fused.down.consume_weight_grad(), "gw_d")):
        gb = bf16_bits(got)
        assert_close_rel(O.bf16_bits_to_f32(gb), O.bf16_bits_to_f32(want[key]), 1e-3, what,
                         ulp_bits=gb, ulp_want=want[key])


def test_fused_mlp_three_d_input_and_no_grad():
    fused, plain = _pair(64, 48, seed=3)
    x = torch.randn(2, 5, 64, device=DEV).to(torch.bfloat16)
    with torch.no_grad():
        y = fused(x)
        y2 = plain(x)
    assert y.shape == (2, 5, 64)
    np.testing.assert_array_equal(bf16_bits(y), bf16_bits(y2))
    with pytest.raises(ValueError):
        fused(torch.randn(3, 65, device=DEV))


def test_full_size_fused_kernels_equal_unfused():
    """At the benchmark's shapes (T=8192, d=4096, f=11008): the gate/up GEMM with h in its
    epilogue equals the GEMM followed by the quantiser, the backward quantiser equals torch's
    autograd followed by the plain dual quantiser, and the dh GEMM with the backward in its
    epilogue equals the GEMM followed by the backward quantiser, bit for bit."""
    T, Fh, K = 8192, 11008, 4096
    gen = torch.Generator(device=DEV).manual_seed(2024)
    a = torch.randint(-127, 128, (T, K), dtype=torch.int8, device=DEV, generator=gen)
    w = torch.randint(-127, 128, (2 * Fh, K), dtype=torch.int8, device=DEV, generator=gen)
    sa = torch.rand(T, device=DEV, generator=gen) * 2e-4 + 1e-5
    sb = torch.rand(2 * Fh, device=DEV, generator=gen) * 2e-3 + 1e-4
    gu_ref = _capi.gemm_i8(a, w, K, scale_a=sa, scale_b=sb, out_kind=_capi.FF_OUT_BF16)
    want = _capi.swiglu_quant(gu_ref)
    gu, *got = _capi.swiglu_gemm(a, w, K, sa, sb)
    assert torch.equal(gu.view(torch.int16), gu_ref.view(torch.int16))
    assert torch.equal(got[4].view(torch.int16), want[4].view(torch.int16))
    for x, y in zip(got[:4], want[:4]):
        assert torch.equal(x, y)
    del a, w, gu, got, want
    g = gu_ref.detach().requires_grad_(True)
    dh = torch.randn(T, Fh, device=DEV, generator=gen).to(torch.bfloat16)
    cm = torch.rand(2 * Fh, device=DEV, generator=gen) * 1e-3
    gg, uu = g.chunk(2, dim=1)
    (F.silu(gg) * uu).backward(dh)
    want = _capi.quant_dual(g.grad, row_colmul=cm)
    got = _capi.swiglu_bwd_quant(dh, gu_ref, colmul=cm)
    assert torch.equal(got[4].view(torch.int16), g.grad.view(torch.int16))
    for x, y in zip(got[:4], want[:4]):
        assert torch.equal(x, y)
    del g, got, want
    # the dh GEMM (K = 4096 -> F) with the backward in its epilogue
    a = torch.randint(-127, 128, (T, K), dtype=torch.int8, device=DEV, generator=gen)
    wd = torch.randint(-127, 128, (K, Fh), dtype=torch.int8, device=DEV, generator=gen)
    sg = torch.rand(T, device=DEV, generator=gen) * 1e-4
    dh = _capi.gemm_i8(a, wd, K, scale_a=sg, out_kind=_capi.FF_OUT_BF16, b_kn_cols=Fh)
    want = _capi.swiglu_bwd_quant(dh, gu_ref, colmul=cm)
    got = _capi.swiglu_bwd_gemm(a, wd, K, sg, gu_ref, colmul=cm)
    assert torch.equal(got[4].view(torch.int16), want[4].view(torch.int16))
    for x, y in zip(got[:4], want[:4]):
        assert torch.equal(x, y)
    assert _capi.device_status() == 0


def test_fused_mlp_empty_batch():
    fused, _ = _pair(64, 128, seed=5)
    x = torch.zeros(0, 64, device=DEV, dtype=torch.bfloat16).requires_grad_(True)
    y = fused(x)
    assert y.shape == (0, 64)
    y.sum().backward()
    assert x.grad.shape == (0, 64)
    gw = fused.gate_up.consume_weight_grad()
    assert gw.shape == (256, 64) and not gw.any()
