"""Pin the CPU oracle to fixtures produced by running the reference (tests/golden/make_golden.py)."""
import numpy as np
import pytest

from oracle import firefly_oracle as O
from tests._util import check_optim_step, load_golden


def _golden_cases(z, suffix):
    return sorted({k[: -len(suffix)] for k in z.files if k.endswith(suffix)})


def test_quantize_rows_bit_exact():
    z = load_golden("quant_rows.npz")
    cases = _golden_cases(z, "_q")
    assert {"normal", "edges", "ties", "bf16", "onecol", "eps"} <= set(cases)
    for c in cases:
        eps = 1e-5 if c == "eps" else 1e-8
        q, s = O.quantize_rows(z[c + "_x"], eps=eps)
        np.testing.assert_array_equal(q, z[c + "_q"], err_msg=c)
        np.testing.assert_array_equal(s.view(np.uint32), z[c + "_s"].view(np.uint32), err_msg=c)


def test_quantize_rows_rejects_non_2d_and_empty_rows():
    with pytest.raises(ValueError):
        O.quantize_rows(np.zeros(5, np.float32))
    with pytest.raises(ValueError):
        O.quantize_rows(np.zeros((3, 0), np.float32))
    q, s = O.quantize_rows(np.zeros((0, 7), np.float32))
    assert q.shape == (0, 7) and s.shape == (0,)


def test_mulaw_codecs():
    z = load_golden("mulaw.npz")
    for c in "abcd":
        x, bs = z[c + "_x"], int(z[c + "_bs"])
        qs, a = O.encode_signed(x, bs)
        np.testing.assert_array_equal(qs, z[c + "_qs"])
        np.testing.assert_array_equal(a, z[c + "_as"])
        qu, au = O.encode_unsigned(x * x, bs)
        np.testing.assert_array_equal(qu, z[c + "_qu"])
        np.testing.assert_array_equal(au, z[c + "_au"])
        # decode: the oracle rounds exp correctly, torch's CPU exp is within an ulp
        for dec, key, qk, ak in ((O.decode_signed, "_ds", "_qs", "_as"), (O.decode_unsigned, "_du", "_qu", "_au")):
            got = dec(z[c + qk], z[c + ak], bs)
            want = z[c + key]
            np.testing.assert_allclose(got, want, rtol=3e-7, atol=0)


def test_decode_tables_within_a_few_ulps():
    # exp(t) - 1 cancels for small t, so one ulp of exp can become a few ulps of x_norm
    z = load_golden("mulaw.npz")
    for got, want in ((O.decode_table_signed(), z["table_signed"]), (O.decode_table_unsigned(), z["table_unsigned"])):
        ulps = np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64))
        assert ulps.max() <= 4 and (ulps > 0).sum() <= 8


def test_zero_state_encoding():
    st = O.init_state((3, 100))
    assert (st["m_q"] == 128).all() and (st["v_q"] == 0).all() and (st["r_q"] == 128).all()
    assert st["m_absmax"].shape == (2,) and np.all(st["m_absmax"] == np.float32(1e-12))


@pytest.mark.parametrize("case", ["cfg1like", "ragged", "defaultwd", "unbiased", "bigstep"])
def test_optimizer_step_matches_reference(case):
    """Replay each recorded step from the recorded previous state with the recorded uniforms."""
    z = load_golden("optim_step.npz")
    O_, K, bs = (int(v) for v in z[case + "_meta"])
    lr, b1, b2, eps, wd, sr = (float(v) for v in z[case + "_hyper"])
    ws = z[case + "_ws"]
    q = z[case + "_q0"]
    st = O.init_state((O_, K), bs)
    keys = ("m_q", "m_absmax", "v_q", "v_absmax", "r_q", "r_absmax")
    for s in range(3):
        g = O.bf16_bits_to_f32(z[f"{case}_s{s}_g"])
        qn, stn = O.dqt_adamw8_step(q, ws, g, st, lr=lr, beta1=b1, beta2=b2, eps=eps, wd=wd,
                                    sr_bias=sr, bs=bs, u=z[f"{case}_s{s}_u"])
        want = {k: z[f"{case}_s{s}_{k}"] for k in keys}
        # rows whose weight_scale is below eps divide by eps=1e-8: the residual there is
        # ill-conditioned (an ulp of adam moves it by ~1e-1 codes), so its codes are
        # compared on the well-conditioned rows only; the int8 weight is compared everywhere
        good = np.asarray(ws) > eps
        np.testing.assert_array_equal(qn, z[f"{case}_s{s}_q"], err_msg=f"{case} step {s}")
        rows = np.nonzero(good)[0]
        sub_got = {k: (stn[k][rows] if stn[k].shape == (O_, K) else stn[k]) for k in keys}
        sub_want = {k: (want[k][rows] if want[k].shape == (O_, K) else want[k]) for k in keys}
        check_optim_step(qn[rows], sub_got, z[f"{case}_s{s}_q"][rows], sub_want, f"{case} step {s}")
        q = z[f"{case}_s{s}_q"]
        st = {"step": s + 1, **want}


def test_int8_linear_close_to_live_bf16_reference():
    """Accuracy figure: the int8 path against the reference's live bf16 path (not a parity gate)."""
    z = load_golden("linear_bf16.npz")
    for c in ("fp32", "bias_bf16"):
        x, q, s = z[c + "_x"], z[c + "_q"], z[c + "_s"]
        bias = z[c + "_bias"] if z[c + "_bias"].size else None
        y_bits, *_ = O.linear_forward(x, q, s, bias)
        y = O.bf16_bits_to_f32(y_bits)
        y_ref = O.bf16_bits_to_f32(z[c + "_y"])
        rel = np.linalg.norm(y - y_ref) / np.linalg.norm(y_ref)
        assert rel < 0.02, (c, rel)
        out = O.linear_backward(x, z[c + "_dy"], q, s, has_bias=bias is not None)
        # the fixture ran forward+backward twice: x.grad and the grad cache hold 2x one pass
        dx = 2 * O.bf16_bits_to_f32(out["dx"])
        assert np.linalg.norm(dx - z[c + "_dx"]) / np.linalg.norm(z[c + "_dx"]) < 0.03
        gw2 = O.bf16_bits_to_f32(O.f32_to_bf16_bits(O.bf16_bits_to_f32(out["gw"]) * 2))
        want = O.bf16_bits_to_f32(z[c + "_gw2"])
        assert np.linalg.norm(gw2 - want) / np.linalg.norm(want) < 0.03


def test_philox_known_answer():
    """Philox4x32-10 known-answer vectors (Random123 distribution, kat_vectors)."""
    out = O.philox4x32_10(np.uint32(0), np.uint32(0), np.uint32(0), np.uint32(0), np.uint32(0), np.uint32(0))
    assert [int(v) for v in out] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    f = np.uint32(0xFFFFFFFF)
    out = O.philox4x32_10(f, f, f, f, f, f)
    assert [int(v) for v in out] == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    out = O.philox4x32_10(np.uint32(0x243F6A88), np.uint32(0x85A308D3), np.uint32(0x13198A2E),
                          np.uint32(0x03707344), np.uint32(0xA4093822), np.uint32(0x299F31D0))
    assert [int(v) for v in out] == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_philox_uniforms_layout():
    u = O.philox_uniforms(64, seed=7, step=3, elem_offset=16)
    assert u.shape == (64,) and u.dtype == np.float32
    assert (u > 0).all() and (u < 1).all()
    # the same global elements give the same draws whatever the offset of the request
    u2 = O.philox_uniforms(32, seed=7, step=3, elem_offset=48)
    np.testing.assert_array_equal(u[32:], u2)
    assert not np.array_equal(O.philox_uniforms(8, 7, 4), O.philox_uniforms(8, 7, 3))


# --------------------------------------------------------------------------
# BitLinear construction (bitLinear.py:15-27, :40-66)
# --------------------------------------------------------------------------
def test_kaiming_draw_quantised_by_oracle_matches_reference_init():
    """The reference's ``BitLinear(K, O)`` under ``torch.manual_seed(s)``: a Kaiming-uniform draw of
    torch's default CPU generator, quantised per row.  The oracle's quantiser on the same draw gives
    the reference's buffers bit for bit, and the construction consumed exactly that draw."""
    import math

    import torch

    z = load_golden("bitlinear_init.npz")
    cases = _golden_cases(z, "_meta")
    assert len(cases) >= 4
    for c in cases:
        K, O_, seed = (int(v) for v in z[c + "_meta"])
        torch.manual_seed(seed)
        w = torch.empty((O_, K), dtype=torch.float32)
        torch.nn.init.kaiming_uniform_(w, a=math.sqrt(5))
        nxt = torch.rand(4).numpy()
        q, s = O.quantize_rows(w.numpy())
        np.testing.assert_array_equal(q, z[c + "_q"], err_msg=c)
        np.testing.assert_array_equal(s.view(np.uint32), z[c + "_s"].view(np.uint32), err_msg=c)
        np.testing.assert_array_equal(nxt, z[c + "_next"], err_msg=c)


# --------------------------------------------------------------------------
# The torch restatement of the reference's live path (the CPU baseline)
# --------------------------------------------------------------------------
def test_ref_torch_linear_equals_reference():
    """``oracle.ref_torch`` forward/backward (fireflykernels.py:164-210) on the recorded inputs, run
    twice like the fixture (the grad cache accumulates): y, dX, dW and db equal the reference's bits."""
    import torch

    from oracle import ref_torch as R
    from tests._util import from_bf16_bits

    z = load_golden("linear_bf16.npz")
    for c in ("fp32", "bias_bf16"):
        xdt = torch.bfloat16 if bool(z[c + "_xisbf16"]) else torch.float32
        x = torch.from_numpy(z[c + "_x"]).to(xdt).requires_grad_(True)
        q, s = torch.from_numpy(z[c + "_q"]), torch.from_numpy(z[c + "_s"])
        bias = torch.from_numpy(z[c + "_bias"]).requires_grad_(True) if z[c + "_bias"].size else None
        dy = from_bf16_bits(z[c + "_dy"])
        cache = {}
        for _ in range(2):
            y = R._LinearFn.apply(x, q, s, bias, cache, 1)
            y.backward(dy)
        np.testing.assert_array_equal(y.detach().view(torch.int16).numpy().view(np.uint16), z[c + "_y"], err_msg=c)
        np.testing.assert_array_equal(x.grad.float().numpy(), z[c + "_dx"], err_msg=c)
        np.testing.assert_array_equal(cache[1].view(torch.int16).numpy().view(np.uint16), z[c + "_gw2"], err_msg=c)
        if bias is not None:
            np.testing.assert_array_equal(bias.grad.numpy(), z[c + "_db2"], err_msg=c)


@pytest.mark.parametrize("case", ["cfg1like", "ragged", "defaultwd", "unbiased", "bigstep"])
def test_ref_torch_optimizer_step_equals_reference(case):
    """``oracle.ref_torch.dqt_step`` (fireflyoptim.py:136-209) from the reference's zero state, fed the
    recorded gradients and uniforms, reproduces every recorded weight, code and absmax exactly."""
    import torch

    from oracle import ref_torch as R
    from tests._util import from_bf16_bits

    z = load_golden("optim_step.npz")
    O_, K, bs = (int(v) for v in z[case + "_meta"])
    lr, b1, b2, eps, wd, sr = (float(v) for v in z[case + "_hyper"])
    q = torch.from_numpy(z[case + "_q0"].copy())
    ws = torch.from_numpy(z[case + "_ws"])
    st = R.init_state((O_, K), bs=bs)
    for s in range(3):
        R.dqt_step(q, ws, from_bf16_bits(z[f"{case}_s{s}_g"]), st, lr=lr, beta1=b1, beta2=b2, eps=eps, wd=wd,
                   sr_bias=sr, bs=bs, u=torch.from_numpy(z[f"{case}_s{s}_u"]))
        np.testing.assert_array_equal(q.numpy(), z[f"{case}_s{s}_q"], err_msg=f"{case} step {s}")
        for k in ("m_q", "m_absmax", "v_q", "v_absmax", "r_q", "r_absmax"):
            np.testing.assert_array_equal(st[k].numpy(), z[f"{case}_s{s}_{k}"], err_msg=f"{case} step {s} {k}")
        assert st["step"] == s + 1
