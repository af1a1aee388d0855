"""BitLinear forward/backward through the int8 tensor-core path against the oracle."""
import numpy as np
import pytest
import torch

import firefly_b200 as ff
from firefly_b200 import fireflykernels as fk
from oracle import firefly_oracle as O
from tests._util import assert_close_rel, bf16_bits, bf16_ulp_diff, check_optim_step, from_bf16_bits, load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
REL = 1e-3


def _layer(K, O_, bias, seed):
    torch.manual_seed(seed)
    layer = ff.BitLinear(K, O_, bias=bias)
    w = torch.randn(O_, K, generator=torch.Generator().manual_seed(seed)) * 0.02
    q, s = ff.quantize_fp_to_int8(w)
    layer.int_weight.copy_(q)
    layer.weight_scale.copy_(s)
    if bias:
        with torch.no_grad():
            layer.bias.copy_(torch.randn(O_, generator=torch.Generator().manual_seed(seed + 1)) * 0.1)
    return layer.to(DEV)


@pytest.mark.parametrize("T,K,O_,bias,xdt", [
    (256, 1024, 1024, False, torch.float32),   # the single-layer config
    (48, 64, 32, True, torch.bfloat16),
    (37, 100, 70, True, torch.float32),        # K and O not multiples of 16, ragged T
    (1, 16, 16, False, torch.bfloat16),
])
def test_forward_backward_match_oracle(T, K, O_, bias, xdt):
    layer = _layer(K, O_, bias, seed=T + K)
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(T, K, generator=g)).to(xdt)
    dy = torch.randn(T, O_, generator=g).to(torch.bfloat16)
    xd = x.to(DEV).requires_grad_(True)
    y = layer(xd)
    assert y.dtype == torch.bfloat16 and y.shape == (T, O_)
    y.backward(dy.to(DEV))
    q = layer.int_weight.cpu().numpy()
    s = layer.weight_scale.cpu().numpy()
    b = layer.bias.detach().cpu().numpy() if bias else None
    y_o, *_ = O.linear_forward(x.float().numpy(), q, s, b)
    # same fp32 epilogue as the oracle: bf16 outputs identical
    np.testing.assert_array_equal(bf16_bits(y), y_o)
    out = O.linear_backward(x.float().numpy(), bf16_bits(dy), q, s, has_bias=bias)
    assert xd.grad.dtype == xdt
    np.testing.assert_array_equal(bf16_bits(xd.grad.to(torch.bfloat16)), out["dx"])
    gw = layer.consume_weight_grad()
    assert gw.dtype == torch.bfloat16 and gw.shape == (O_, K)
    np.testing.assert_array_equal(bf16_bits(gw), out["gw"])
    assert layer.consume_weight_grad() is None
    if bias:
        assert bf16_ulp_diff(bf16_bits(layer.bias.grad), out["db"]).max() <= 1


def test_grad_cache_accumulates_across_micro_batches():
    layer = _layer(96, 80, False, seed=1)
    g = torch.Generator().manual_seed(2)
    xs = [torch.randn(64, 96, generator=g) for _ in range(2)]
    dys = [torch.randn(64, 80, generator=g).to(torch.bfloat16) for _ in range(2)]
    cache = None
    q, s = layer.int_weight.cpu().numpy(), layer.weight_scale.cpu().numpy()
    for x, dy in zip(xs, dys):
        y = layer(x.to(DEV).requires_grad_(True))
        y.backward(dy.to(DEV))
        out = O.linear_backward(x.numpy(), bf16_bits(dy), q, s, grad_cache=cache)
        cache = out["gw"]
    np.testing.assert_array_equal(bf16_bits(layer.consume_weight_grad()), cache)


def test_three_d_input_and_errors():
    layer = _layer(32, 48, False, seed=3)
    x = torch.randn(2, 5, 32, device=DEV)
    y = layer(x)
    assert y.shape == (2, 5, 48)
    with pytest.raises(ValueError):
        layer(torch.randn(4, 31, device=DEV))
    with pytest.raises(RuntimeError):
        layer(torch.randn(4, 32))  # CPU input, CUDA module
    # no-grad forward does not leave a gradient behind
    with torch.no_grad():
        layer(x)
    assert layer.consume_weight_grad() is None


def test_accuracy_against_live_bf16_reference():
    """The reference computes in bf16 (fireflykernels.py:164-210); the int8 path stays close."""
    z = load_golden("linear_bf16.npz")
    for c in ("fp32", "bias_bf16"):
        x = torch.from_numpy(z[c + "_x"])
        if bool(z[c + "_xisbf16"]):
            x = x.to(torch.bfloat16)
        q, s = torch.from_numpy(z[c + "_q"]), torch.from_numpy(z[c + "_s"])
        O_, K = q.shape
        layer = ff.BitLinear(K, O_, bias=bool(z[c + "_bias"].size)).to(DEV)
        layer.int_weight.copy_(q)
        layer.weight_scale.copy_(s)
        if layer.bias is not None:
            with torch.no_grad():
                layer.bias.copy_(torch.from_numpy(z[c + "_bias"]))
        y = layer(x.to(DEV))
        y_ref = from_bf16_bits(z[c + "_y"]).float()
        rel = (y.float().cpu() - y_ref).norm() / y_ref.norm()
        assert rel < 0.02, (c, float(rel))


def test_state_dict_reregisters_handle():
    a = _layer(16, 16, False, seed=4)
    b = _layer(16, 16, False, seed=5)
    ha, hb = a._registered_handle, b._registered_handle
    assert ha != hb
    b.load_state_dict(a.state_dict())
    assert b._registered_handle == ha
    assert hb not in fk._REGISTERED_HANDLES
    assert torch.equal(a.int_weight, b.int_weight)


def test_weight_cache_invalidated_by_optimizer():
    """K = 70 is not a multiple of 16: the GEMMs read a padded copy of W, which must follow
    every optimizer update (the role of _invalidate_weight_cache, fireflyoptim.py:198)."""
    layer = _layer(70, 48, False, seed=6)
    x = torch.randn(32, 70, device=DEV, requires_grad=True)
    opt = ff.FireFlyOptim([torch.nn.Parameter(torch.zeros(1, device=DEV))], lr=5e-2, bit_modules=[layer])
    q, s = layer.int_weight.cpu().numpy(), layer.weight_scale.cpu().numpy()
    for _ in range(3):
        y = layer(x)
        dy = torch.randn_like(y)
        y.backward(dy)
        out = O.linear_backward(x.detach().cpu().numpy(), bf16_bits(dy), q, s)
        np.testing.assert_array_equal(bf16_bits(x.grad.to(torch.bfloat16)), out["dx"])
        x.grad = None
        opt.step()
        q = layer.int_weight.cpu().numpy()
        wk = fk._weight_operand(layer._registered_handle, layer.int_weight)
        np.testing.assert_array_equal(wk.cpu().numpy()[:, :70], q)


# --------------------------------------------------------------------------
# Construction and module discovery (bitLinear.py:15-27, :40-66, :107-108; fireflyoptim.py:114-120)
# --------------------------------------------------------------------------
def test_init_matches_reference_construction():
    """``BitLinear(K, O)`` under ``torch.manual_seed(s)`` holds the reference's ``int_weight`` and
    ``weight_scale`` bit for bit (recorded by running the reference's constructor), and draws
    exactly as many numbers from the default generator."""
    z = load_golden("bitlinear_init.npz")
    cases = sorted(k[:-5] for k in z.files if k.endswith("_meta"))
    assert len(cases) >= 4
    for c in cases:
        K, O_, seed = (int(v) for v in z[c + "_meta"])
        torch.manual_seed(seed)
        layer = ff.BitLinear(K, O_)
        nxt = torch.rand(4).numpy()
        assert layer.int_weight.dtype == torch.int8 and layer.int_weight.shape == (O_, K)
        assert layer.weight_scale.dtype == torch.float32 and layer.weight_scale.shape == (O_,)
        np.testing.assert_array_equal(layer.int_weight.numpy(), z[c + "_q"], err_msg=c)
        np.testing.assert_array_equal(layer.weight_scale.numpy().view(np.uint32), z[c + "_s"].view(np.uint32),
                                      err_msg=c)
        np.testing.assert_array_equal(nxt, z[c + "_next"], err_msg=c)
        # reset_int8_ redraws from the generator like the constructor
        torch.manual_seed(seed)
        layer.reset_int8_()
        np.testing.assert_array_equal(layer.int_weight.numpy(), z[c + "_q"], err_msg=c)


def test_collect_and_add_bit_modules():
    a, b = ff.BitLinear(32, 16), ff.BitLinear(16, 8, bias=True)
    net = torch.nn.Sequential(a, torch.nn.GELU(), torch.nn.Sequential(torch.nn.Identity(), b))
    assert ff.collect_bitlinear_modules(net) == [a, b]
    assert ff.collect_bitlinear_modules(torch.nn.Linear(3, 3)) == []
    opt = ff.FireFlyOptim([torch.nn.Parameter(torch.zeros(1))], bit_modules=[a])
    opt.add_bit_modules(ff.collect_bitlinear_modules(net))  # a is already there
    assert opt.bit_modules == [a, b]
    assert opt._bit_handles == [a._registered_handle, b._registered_handle]
    with pytest.raises(TypeError, match="expected BitLinear, got Linear"):
        opt.add_bit_modules([torch.nn.Linear(2, 2)])
    assert opt.bit_modules == [a, b]


def test_fireflyoptim_sr_is_unbiased_rounding():
    """``FireFlyOptimSR`` (fireflyoptim.py:236-258) is ``FireFlyOptim`` with ``sr_bias_scale`` 0: with
    the same uniforms its steps equal the oracle's unbiased update and differ from the biased one."""
    layer = _layer(256, 64, False, seed=8)
    opt = ff.FireFlyOptimSR([torch.nn.Parameter(torch.zeros(1, device=DEV))], lr=5e-3, weight_decay=0.01,
                            bit_modules=[layer])
    assert opt.sr_bias_scale == 0.0 and isinstance(opt, ff.FireFlyOptim)
    rng = np.random.default_rng(8)
    q, ws = layer.int_weight.cpu().numpy(), layer.weight_scale.cpu().numpy()
    st = O.init_state(q.shape)
    us = {}
    opt.uniform_source = lambda m, h, t: torch.from_numpy(us[t])
    h = layer._registered_handle
    biased_differs = False
    for t in range(1, 4):
        g_bits = O.f32_to_bf16_bits(rng.standard_normal(q.shape).astype(np.float32))
        us[t] = rng.random(q.shape, dtype=np.float32)
        fk._BIT_GRAD_CACHE[h] = from_bf16_bits(g_bits, DEV)
        opt.step()
        q_o, st_o = O.dqt_adamw8_step(q, ws, O.bf16_bits_to_f32(g_bits), st, lr=5e-3, wd=0.01, sr_bias=0.0,
                                      u=us[t])
        q_b, _ = O.dqt_adamw8_step(q, ws, O.bf16_bits_to_f32(g_bits), st, lr=5e-3, wd=0.01, sr_bias=0.15,
                                   u=us[t])
        got = {k: v.cpu().numpy() for k, v in opt._bit_state[h].items() if torch.is_tensor(v)}
        check_optim_step(layer.int_weight.cpu().numpy(), got, q_o, st_o, f"SR step {t}")
        biased_differs |= not np.array_equal(q_b, q_o)
        q, st = layer.int_weight.cpu().numpy(), {"step": t, **got}
    assert biased_differs  # the bias term matters on these inputs, so the test can tell them apart


# --------------------------------------------------------------------------
# The activation-code cache
# --------------------------------------------------------------------------
def test_activation_codes_not_reused_across_steps_after_untracked_write():
    """An input buffer rewritten through ``.data`` (which does not bump the version counter that keys
    the activation-code cache) between training steps is quantised afresh: the cache is dropped by
    the backward pass and by the optimizer step."""
    layer = _layer(128, 64, False, seed=9)
    opt = ff.FireFlyOptim([torch.nn.Parameter(torch.zeros(1, device=DEV))], lr=0.0, weight_decay=0.0,
                          bit_modules=[layer])
    g = torch.Generator(device=DEV).manual_seed(9)
    x = torch.randn(32, 128, device=DEV, generator=g).requires_grad_(True)
    x2 = torch.randn(32, 128, device=DEV, generator=g)
    want = layer(x2.clone().requires_grad_(True)).detach()
    y = layer(x)
    y.backward(torch.ones_like(y))
    x.data.copy_(x2)  # untracked write: x._version does not change
    assert torch.equal(layer(x).detach(), want)  # dropped by the backward pass
    with torch.no_grad():
        layer(x)
    opt.step()
    x.data.copy_(x2 * 2)
    with torch.no_grad():
        assert torch.equal(layer(x), layer((x2 * 2).clone()))  # dropped by the optimizer step
