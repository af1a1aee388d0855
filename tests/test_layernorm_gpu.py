"""LayerNorm with the quantiser's first pass folded in (``ff_layernorm_i8``) and its backward
(``ff_layernorm_bwd``), used by the BitLinear decoder.

* the output is within one bf16 step of the fp64 LayerNorm of the same bf16 input (fp32
  arithmetic, then one bf16 rounding), mean and rstd within fp32 accuracy;
* the int8 codes returned with it are exactly ``quant_dual`` of the output;
* dgamma, dbeta and the input gradient of ``LayerNormQuantFn`` agree with fp64 autograd;
* the next BitLinear finds the codes in the activation cache instead of quantising again;
* a decoder with these LayerNorms stays close to the one with torch's.
"""
import pytest
import torch
from torch.nn import functional as F

from firefly_b200 import _capi
from firefly_b200.decoder import DecoderConfig, LayerNormQuantFn, build_decoder, synthetic_batches
from firefly_b200.fireflykernels import _quantize_activation
from tests._util import bf16_bits, bf16_ulp_diff

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _inputs(T, C, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = (torch.randn(T, C, device=DEV, generator=g) * 3 + 0.5).to(torch.bfloat16)
    w = torch.randn(C, device=DEV, generator=g) * 0.5 + 1
    b = torch.randn(C, device=DEV, generator=g) * 0.1
    return x, w, b


def _ref(x, w, b, eps):
    x64 = x.double()
    mu = x64.mean(dim=1, keepdim=True)
    var = ((x64 - mu) ** 2).mean(dim=1, keepdim=True)
    return (x64 - mu) / torch.sqrt(var + eps) * w.double() + b.double(), mu.squeeze(1), (var + eps).rsqrt().squeeze(1)


@pytest.mark.parametrize("T,C", [(1000, 2048), (37, 4096), (513, 264)])
def test_forward_close_to_fp64_and_codes_exact(T, C):
    x, w, b = _inputs(T, C, seed=T + C)
    y, mean, rstd, codes = _capi.layernorm_quant(x, w, b, eps=1e-5)
    ref, mu, rs = _ref(x, w, b, 1e-5)
    # fp32 arithmetic then one bf16 rounding: within a bf16 step of the fp64 value, plus a small
    # absolute floor where (x - mean)*rstd*gamma and beta cancel
    err = (y.double() - ref).abs()
    assert bool((err <= 2.0 ** -8 * ref.abs() + 1e-4).all()), float((err - 2.0 ** -8 * ref.abs()).max())
    ulps = bf16_ulp_diff(bf16_bits(y), bf16_bits(ref.to(torch.bfloat16)))
    assert (ulps > 0).mean() < 0.05, (ulps > 0).mean()
    torch.testing.assert_close(mean.double(), mu, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(rstd.double(), rs, rtol=1e-5, atol=1e-6)
    for name, got, want in zip(("q_rows", "s_rows", "q_cols_t", "s_cols"), codes, _capi.quant_dual(y)):
        assert torch.equal(got, want), name


@pytest.mark.parametrize("T,C", [(1000, 2048), (100, 264)])
def test_backward_agrees_with_fp64_autograd(T, C):
    x, w, b = _inputs(T, C, seed=3 * T + C)
    wp, bp = w.clone().requires_grad_(True), b.clone().requires_grad_(True)
    xp = x.clone().requires_grad_(True)
    y = LayerNormQuantFn.apply(xp, wp, bp, 1e-5, True)
    dy = torch.randn(T, C, device=DEV).to(torch.bfloat16)
    y.backward(dy)
    x64 = x.double().requires_grad_(True)
    w64, b64 = w.double().requires_grad_(True), b.double().requires_grad_(True)
    F.layer_norm(x64, (C,), w64, b64, 1e-5).backward(dy.double())
    torch.testing.assert_close(wp.grad.double(), w64.grad, rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(bp.grad.double(), b64.grad, rtol=1e-4, atol=1e-3)
    rel = (xp.grad.double() - x64.grad).norm() / x64.grad.norm()
    assert rel < 1e-2, float(rel)


def test_next_bitlinear_reuses_the_codes():
    x, w, b = _inputs(256, 512, seed=5)
    y = LayerNormQuantFn.apply(x.view(4, 64, 512), w, b, 1e-5, True)
    codes = _quantize_activation(y.reshape(-1, 512), with_cols=True)
    again = _capi.quant_dual(y.reshape(-1, 512))
    for got, want in zip(codes, again):
        assert torch.equal(got, want)
    from firefly_b200.fireflykernels import _ACT_CACHE

    assert _ACT_CACHE["entry"][2] is codes  # the codes registered by the LayerNorm, not a new quantisation


def test_decoder_with_fused_norms_stays_close():
    cfg = DecoderConfig(vocab=512, d_model=256, heads=4, ffn=1024, layers=2, max_seq=64)
    a = build_decoder(cfg, DEV, seed=21, fused=True, fused_norm=True)
    b = build_decoder(cfg, DEV, seed=21, fused=True, fused_norm=False)
    ids, tgt = synthetic_batches(cfg, 2, 64, 2, DEV, seed=22)[0]
    with torch.no_grad():
        la, lb = a(ids).float(), b(ids).float()
    rel = (la - lb).norm() / lb.norm()
    assert rel < 0.02, float(rel)
