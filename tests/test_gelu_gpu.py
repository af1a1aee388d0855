"""GELU producer fusion: the GELU GEMM epilogues and the fused GELU MLP op of the decoder.

* the epilogues' GELU arithmetic equals torch's tanh-form GELU kernels for every bf16 input
  (forward in bf16, the derivative in fp32);
* ``ff_gelu_gemm_i8`` gives exactly the BitLinear up projection's output u, torch's bf16
  ``F.gelu(u, approximate="tanh")`` and ``quant_dual`` of it;
* ``ff_gelu_bwd_gemm_i8`` gives exactly torch's ``gelu_backward`` of the bf16 dh that the dX
  GEMM produces, and ``quant_dual`` of it with the up projection's column multipliers;
* a decoder with the fused op equals the decoder built from BitLinear layers and torch's GELU,
  bit for bit, in the forward and in every weight gradient.
"""
import pytest
import torch
from torch.nn import functional as F

from firefly_b200 import _capi
from firefly_b200.decoder import DecoderConfig, build_decoder, synthetic_batches
from firefly_b200.fireflykernels import _BIT_GRAD_CACHE

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
NAMES = ("q_rows", "s_rows", "q_cols_t", "s_cols")


def _eq(a, b, name):
    assert a.shape == b.shape and a.dtype == b.dtype, name
    if a.is_floating_point():
        assert _capi._same_bits(a.contiguous(), b.contiguous()), name
    else:
        assert torch.equal(a, b), name


def test_gelu_arithmetic_equals_torch_for_every_bf16_input():
    v = _capi.gelu_variant(DEV)
    x = torch.arange(-32768, 32768, dtype=torch.int32, device=DEV).to(torch.int16).view(torch.bfloat16)
    h, d = _capi.gelu_eval(x, v & 1, v & ~1)
    _eq(h.to(torch.bfloat16), F.gelu(x, approximate="tanh"), "gelu")
    ones = torch.ones(x.shape, dtype=torch.float32, device=DEV)
    _eq(d, torch.ops.aten.gelu_backward(ones, x.float(), approximate="tanh"), "gelu'")


def _codes(T, K, F_, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    a = torch.randint(-127, 128, (T, K), dtype=torch.int8, device=DEV, generator=g)
    w = torch.randint(-127, 128, (F_, K), dtype=torch.int8, device=DEV, generator=g)
    sa = torch.rand(T, device=DEV, generator=g) * 2e-3 + 1e-4
    sb = torch.rand(F_, device=DEV, generator=g) * 2e-3 + 1e-4
    return a, w, sa, sb


@pytest.mark.parametrize("T,K,F_,bias", [(300, 256, 1056, False), (1024 + 37, 512, 2048, True), (1, 128, 32, False)])
def test_gelu_gemm_equals_gemm_then_torch_gelu_then_quant(T, K, F_, bias):
    a, w, sa, sb = _codes(T, K, F_, seed=T + F_)
    b = torch.randn(F_, device=DEV) * 0.3 if bias else None
    u, *codes, h = _capi.gelu_gemm(a, w, K, sa, sb, bias=b)
    u_ref = _capi.gemm_i8(a, w, K, scale_a=sa, scale_b=sb, bias=b, out_kind=_capi.FF_OUT_BF16)
    _eq(u, u_ref, "u")
    h_ref = F.gelu(u_ref, approximate="tanh")
    _eq(h, h_ref, "h")
    for name, got, want in zip(NAMES, codes, _capi.quant_dual(h_ref)):
        _eq(got, want, name)


@pytest.mark.parametrize("T,O,F_,colmul", [(300, 256, 1056, True), (1024 + 37, 512, 2048, False), (5, 128, 64, True)])
def test_gelu_bwd_gemm_equals_dx_gemm_then_torch_gelu_backward_then_quant(T, O, F_, colmul):
    g = torch.Generator(device=DEV).manual_seed(7 * T + F_)
    a = torch.randint(-127, 128, (T, O), dtype=torch.int8, device=DEV, generator=g)
    w_down = torch.randint(-127, 128, (O, F_), dtype=torch.int8, device=DEV, generator=g)  # [K, F] row-major
    sa = torch.rand(T, device=DEV, generator=g) * 2e-3 + 1e-4
    u = (torch.randn(T, F_, device=DEV, generator=g) * 2).to(torch.bfloat16)
    cm = torch.rand(F_, device=DEV, generator=g) * 1e-2 if colmul else None
    *codes, du = _capi.gelu_bwd_gemm(a, w_down, O, sa, u, colmul=cm)
    dh = _capi.gemm_i8(a, w_down, O, scale_a=sa, out_kind=_capi.FF_OUT_BF16, b_kn_cols=F_)
    du_ref = torch.ops.aten.gelu_backward(dh, u, approximate="tanh")
    _eq(du, du_ref, "du")
    for name, got, want in zip(NAMES, codes, _capi.quant_dual(du_ref, row_colmul=cm)):
        _eq(got, want, name)


def test_fused_decoder_equals_unfused_decoder():
    cfg = DecoderConfig(vocab=512, d_model=256, heads=4, ffn=1024, layers=2, max_seq=64)
    fused = build_decoder(cfg, DEV, seed=11, fused=True, fused_norm=False)
    plain = build_decoder(cfg, DEV, seed=11, fused=False)
    ids, tgt = synthetic_batches(cfg, 3, 64, 3, DEV, seed=12)[0]
    grads = []
    for model in (fused, plain):
        _BIT_GRAD_CACHE.clear()
        logits = model(ids)
        loss = F.cross_entropy(logits.float().view(-1, cfg.vocab), tgt.reshape(-1))
        loss.backward()
        grads.append((logits.detach(), [_BIT_GRAD_CACHE[m._registered_handle].clone() for m in model.bit_modules()],
                      [p.grad.clone() for p in model.parameters()]))
    _BIT_GRAD_CACHE.clear()
    (lf, wf, pf), (lp, wp, pp) = grads
    _eq(lf, lp, "logits")
    for i, (a, b) in enumerate(zip(wf, wp)):
        _eq(a, b, f"dW of BitLinear {i}")
    for i, (a, b) in enumerate(zip(pf, pp)):
        _eq(a, b, f"grad of dense parameter {i}")
